"""scikit-learn estimators (yabt/sklearn_api.py:250-366) over the device
boosting loop. Same constructor parameters (every ``BoostParams`` field plus
``cat_smoothing``), same target handling: the regressor standardises y
(:356-363), the classifier maps binary labels to {0, 1} and uses one-vs-rest
for more classes (:307-331); predict_proba is expit / softmax of the margins.
"""

from __future__ import annotations

from dataclasses import fields

import numpy as np
from scipy.special import expit
from sklearn.base import BaseEstimator, ClassifierMixin, RegressorMixin

from .boosting import Booster, BoostParams, LogLoss, MSELoss
from .multiclass import MulticlassBooster

_PARAM_NAMES = [f.name for f in fields(BoostParams)]


def _require_single_target(y: np.ndarray) -> np.ndarray:
    if y.ndim == 2 and y.shape[1] == 1:
        return y.ravel()
    if y.ndim > 1:
        raise ValueError(f"y has shape {y.shape}; this estimator predicts a single target.")
    return y


class _YABTBase(BaseEstimator):
    def __init__(self, **kwargs):
        defaults = BoostParams()
        for name in _PARAM_NAMES:
            setattr(self, name, kwargs.pop(name, getattr(defaults, name)))
        self.cat_smoothing = kwargs.pop("cat_smoothing", 10.0)
        if kwargs:
            raise TypeError(f"Unknown parameters: {sorted(kwargs)}")

    @classmethod
    def _get_param_names(cls):
        return sorted(_PARAM_NAMES + ["cat_smoothing"])

    def _boost_params(self) -> BoostParams:
        return BoostParams(**{n: getattr(self, n) for n in _PARAM_NAMES})

    @staticmethod
    def _check_cats(categorical_features):
        if categorical_features:
            raise NotImplementedError("categorical target encoding is host preprocessing outside the "
                                      "GPU tree-growth path; encode categorical columns before fit")

    def fit(self, X, y, eval_set=None, categorical_features=None, comm=None):
        """``comm`` (a ``yabt_b200.distributed.ShardComm``): X and y are this
        rank's rows of a row-sharded training set; every rank calls ``fit``
        with the same parameters and ends with the same model."""
        self._check_cats(categorical_features)
        y = _require_single_target(np.asarray(y, dtype=np.float32))
        yt = self._transform_y(y, fit=True, comm=comm)
        ev = None
        if eval_set is not None:
            ev = (eval_set[0], self._transform_y(np.asarray(eval_set[1], dtype=np.float32), fit=False))
        self.booster_ = Booster(self._boost_params(), self._loss())
        self.booster_.fit(X, yt, eval_set=ev, comm=comm)
        return self

    def _margin(self, X) -> np.ndarray:
        return self.booster_.predict_margin(X)


class YABTClassifier(_YABTBase, ClassifierMixin):
    """Binary and multiclass classifier (one-vs-rest for multiclass)."""

    def fit(self, X, y, eval_set=None, categorical_features=None, comm=None):
        """``comm``: row-sharded fit (binary targets), as for YABTRegressor.fit."""
        self._check_cats(categorical_features)
        y = np.asarray(y, dtype=np.float32)
        self.classes_ = np.unique(y)
        if comm is not None:
            import torch
            u = torch.from_numpy(self.classes_.reshape(1, -1).astype(np.float32))
            self.classes_ = np.unique(comm.gather_columns(u).numpy())
        self.n_classes_ = len(self.classes_)
        self._is_binary = self.n_classes_ == 2
        if self._is_binary:
            yt = (y == self.classes_[1]).astype(np.float32)
            ev = None
            if eval_set is not None:
                ye = (np.asarray(eval_set[1], dtype=np.float32) == self.classes_[1]).astype(np.float32)
                ev = (eval_set[0], ye)
            self.booster_ = Booster(self._boost_params(), LogLoss())
            self.booster_.fit(X, yt, eval_set=ev, comm=comm)
        elif comm is not None:
            raise NotImplementedError("row-sharded fits support binary classification only")
        else:
            self.booster_ = MulticlassBooster(self._boost_params())
            self.booster_.fit(X, y, eval_set=eval_set)
        return self

    def predict_proba(self, X) -> np.ndarray:
        if self._is_binary:
            p = expit(self.booster_.predict_margin(X))
            return np.stack([1 - p, p], axis=1)
        return self.booster_.predict_proba(X)

    def predict(self, X) -> np.ndarray:
        if self._is_binary:
            return self.classes_[(self.booster_.predict_margin(X) > 0).astype(int)]
        return self.booster_.predict(X)


class YABTRegressor(_YABTBase, RegressorMixin):
    """Regressor; standardises the target internally."""

    def _loss(self):
        return MSELoss()

    def _transform_y(self, y, fit, comm=None):
        if fit and comm is None:
            self._y_mean = float(y.mean())
            self._y_std = float(y.std()) or 1.0
        elif fit:
            n = sum(comm.int_values(len(y)))
            mean = comm.sum_float(float(y.astype(np.float64).sum())) / n
            var = comm.sum_float(float(((y.astype(np.float64) - mean) ** 2).sum())) / n
            self._y_mean = float(np.float32(mean))
            self._y_std = float(np.float32(np.sqrt(var))) or 1.0
        return (y - self._y_mean) / self._y_std

    def predict(self, X) -> np.ndarray:
        return self._margin(X) * self._y_std + self._y_mean


class YABTMultiTaskRegressor(_YABTBase, RegressorMixin):
    """Multi-output regression with one shared tree structure across the
    targets and a leaf value per target (yabt/sklearn_api.py:366-402): every
    target is standardised, splits are chosen on the summed per-target gain.
    Only the core split and sampling parameters apply, as in the reference."""

    def fit(self, X, Y, eval_set=None):
        from .multitask import MultiTaskBooster
        Y = np.asarray(Y, dtype=np.float32)
        self._y_1d = Y.ndim == 1
        if self._y_1d:
            Y = Y[:, None]
        self.n_tasks_ = Y.shape[1]
        self._y_mean = Y.mean(axis=0)
        std = Y.std(axis=0)
        self._y_std = np.where(std == 0, 1.0, std).astype(np.float32)
        Yt = (Y - self._y_mean) / self._y_std
        ev = None
        if eval_set is not None:
            Yv = np.asarray(eval_set[1], dtype=np.float32)
            if Yv.ndim == 1:
                Yv = Yv[:, None]
            ev = (np.asarray(eval_set[0], dtype=np.float32), (Yv - self._y_mean) / self._y_std)
        self.booster_ = MultiTaskBooster(self._boost_params(), MSELoss())
        self.booster_.fit(np.asarray(X, dtype=np.float32), Yt, eval_set=ev)
        return self

    def predict(self, X) -> np.ndarray:
        m = self.booster_.predict_margin(np.asarray(X, dtype=np.float32))
        out = m * self._y_std + self._y_mean
        return out[:, 0] if self._y_1d else out
