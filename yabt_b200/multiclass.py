"""One-vs-rest multiclass boosting (yabt/multiclass.py:9-48).

Each class gets an independent logistic ``Booster``. Unlike the reference,
which refits an identical Binner for every class, the device matrix (binner,
bin matrix, imputed features) is prepared once and shared by all classes.
"""

from __future__ import annotations

import numpy as np
import torch

from .boosting import Booster, BoostParams, DeviceData, LogLoss


class MulticlassBooster:
    def __init__(self, params: BoostParams):
        self.params = params
        self.boosters_: list[Booster] = []
        self.classes_: np.ndarray | None = None

    def fit(self, X, y, eval_set=None) -> "MulticlassBooster":
        self.classes_ = np.unique(y)
        dev = torch.device(self.params.resolve_device())
        data = DeviceData(X, self.params.max_bins, dev)
        self.boosters_ = []
        for c in self.classes_:
            yb = (np.asarray(y) == c).astype(np.float32)
            ev = None
            if eval_set is not None:
                ev = (eval_set[0], (np.asarray(eval_set[1]) == c).astype(np.float32))
            b = Booster(self.params, LogLoss())
            b.fit(X, yb, eval_set=ev, data=data)
            self.boosters_.append(b)
        return self

    def predict_margin(self, X) -> np.ndarray:
        """Per-class raw scores, (n_samples, n_classes)."""
        return np.stack([b.predict_margin(X) for b in self.boosters_], axis=1)

    def predict_proba(self, X) -> np.ndarray:
        m = self.predict_margin(X)
        e = np.exp(m - m.max(axis=1, keepdims=True))
        return e / e.sum(axis=1, keepdims=True)

    def predict(self, X) -> np.ndarray:
        return self.classes_[np.argmax(self.predict_proba(X), axis=1)]
