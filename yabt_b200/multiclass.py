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

    def fit(self, X, y, eval_set=None, round_callback=None) -> "MulticlassBooster":
        """One boosting round = one tree per class. The class boosters run on
        their own CUDA streams, interleaved tree by tree, so one class's small
        per-level kernels overlap another's histograms. ``round_callback(r)``,
        if given, is called after round r's launches are queued."""
        self.classes_ = np.unique(y)
        dev = torch.device(self.params.resolve_device())
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        data = DeviceData(X, self.params.max_bins, dev)
        main = torch.cuda.current_stream(dev)
        self.boosters_, steps, streams = [], [], []
        for c in self.classes_:
            yb = (np.asarray(y) == c).astype(np.float32)
            ev = None
            if eval_set is not None:
                ev = (eval_set[0], (np.asarray(eval_set[1]) == c).astype(np.float32))
            b = Booster(self.params, LogLoss())
            b._level_wait = False                 # one host thread feeds every stream: never block on one
            st = torch.cuda.Stream(dev)
            st.wait_stream(main)                  # the shared device data is ready
            self.boosters_.append(b)
            steps.append(b.fit_steps(X, yb, eval_set=ev, data=data))
            streams.append(st)
        live = list(range(len(steps)))
        r = 0
        while live:
            for i in list(live):
                with torch.cuda.stream(streams[i]):
                    try:
                        next(steps[i])
                    except StopIteration:
                        live.remove(i)
            if round_callback is not None and live:
                round_callback(r, streams)
            r += 1
        for st in streams:
            main.wait_stream(st)
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
