"""Point methods of the prediction study (rlccl/prediction/models.py).

* ``ewma_history_predictions`` / ``select_recent_backbone`` (mean
  validation RMSE; ties go to the MLP);
* ``RidgeMultiOutput`` (standardised closed-form ridge, moment-only head);
* ``RecentHistoryMLP``: scikit-learn MLPRegressor (32 tanh units, Adam,
  alpha 1e-4, batch 256, 80 epochs, fixed seed) on flattened histories;
* ``NumpyCausalTCN``: one left-padded causal Conv1D layer (kernel 3, 8
  channels, tanh), a head on [last hidden, mean hidden], MSE + L2, Adam
  with bias correction, Glorot-uniform init from the seed.  The
  convolution is a sum of K shifted [B*T, C] x [C, H] products (no per-
  position loop) and its gradient the matching transposed products;
* ``HistoryPredictorSuite``: all six point methods fit on the fit split
  with fit-split standardisation of the recent-history inputs and targets.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any, Mapping

import numpy as np

METHOD_NAMES = ("long_term_mean", "previous_value", "ewma", "moment_only", "recent_history_mlp", "causal_tcn",
                "quantile_scenario")


def ewma_history_predictions(summaries: np.ndarray, alpha: float = 0.30) -> np.ndarray:
    """Post-update EWMA states; the prediction for t uses state t-1."""
    v = np.asarray(summaries, dtype=np.float64)
    if v.ndim != 2 or not len(v):
        raise ValueError("summaries must be a nonempty 2-D array")
    if not 0.0 < alpha <= 1.0:
        raise ValueError("alpha must be in (0, 1]")
    from .data import ewma_rows
    return ewma_rows(v, float(alpha))


def select_recent_backbone(validation_sequence_rmse: Mapping[str, np.ndarray]) -> str:
    want = {"recent_history_mlp", "causal_tcn"}
    if set(validation_sequence_rmse) != want:
        raise ValueError(f"validation scores must contain exactly {sorted(want)}")
    means = {}
    for k, v in validation_sequence_rmse.items():
        a = np.asarray(v, dtype=np.float64).reshape(-1)
        if not len(a) or not np.isfinite(a).all():
            raise ValueError(f"validation scores for {k} must be nonempty and finite")
        means[k] = float(a.mean())
    d = means["recent_history_mlp"] - means["causal_tcn"]
    return "recent_history_mlp" if abs(d) <= 1e-12 or d < 0.0 else "causal_tcn"


@dataclass
class RidgeMultiOutput:
    alpha: float = 10.0
    x_mean: np.ndarray | None = None
    x_scale: np.ndarray | None = None
    y_mean: np.ndarray | None = None
    weights: np.ndarray | None = None

    def fit(self, x, y) -> "RidgeMultiOutput":
        X, Y = np.asarray(x, dtype=np.float64), np.asarray(y, dtype=np.float64)
        if X.ndim != 2 or Y.ndim != 2 or len(X) != len(Y) or not len(X):
            raise ValueError("x and y must be nonempty same-length 2-D arrays")
        self.x_mean = X.mean(axis=0)
        s = X.std(axis=0, ddof=0)
        self.x_scale = np.where(s < 1e-8, 1.0, s)
        Z = (X - self.x_mean) / self.x_scale
        self.y_mean = Y.mean(axis=0)
        self.weights = np.linalg.solve(Z.T @ Z + float(self.alpha) * np.eye(Z.shape[1]), Z.T @ (Y - self.y_mean))
        return self

    def predict(self, x) -> np.ndarray:
        if self.weights is None:
            raise RuntimeError("RidgeMultiOutput is not fitted")
        X = np.asarray(x, dtype=np.float64)
        if X.ndim != 2 or X.shape[1] != self.x_mean.shape[0]:
            raise ValueError("ridge feature shape mismatch")
        return (X - self.x_mean) / self.x_scale @ self.weights + self.y_mean


class RecentHistoryMLP:
    def __init__(self, input_dim: int, output_dim: int, *, seed: int = 20260731,
                 hidden_layer_sizes: tuple[int, ...] = (32,), activation: str = "tanh", solver: str = "adam",
                 alpha: float = 1e-4, batch_size: int = 256, learning_rate_init: float = 1e-3, max_iter: int = 80):
        self.input_dim, self.output_dim, self.seed = int(input_dim), int(output_dim), int(seed)
        self.hidden_layer_sizes, self.activation, self.solver = tuple(hidden_layer_sizes), activation, solver
        self.alpha, self.batch_size = float(alpha), int(batch_size)
        self.learning_rate_init, self.max_iter = float(learning_rate_init), int(max_iter)
        self.early_stopping = False
        self._model: Any | None = None

    def _x(self, x) -> np.ndarray:
        v = np.asarray(x, dtype=np.float64)
        if v.ndim > 2:
            v = v.reshape(len(v), -1)
        if v.ndim != 2 or v.shape[1] != self.input_dim:
            raise ValueError("MLP input dimension mismatch")
        return v

    def fit(self, x, y) -> "RecentHistoryMLP":
        import warnings

        from sklearn.exceptions import ConvergenceWarning
        from sklearn.neural_network import MLPRegressor
        X, Y = self._x(x), np.asarray(y, dtype=np.float64)
        if Y.shape != (len(X), self.output_dim):
            raise ValueError("MLP target dimension mismatch")
        self._model = MLPRegressor(hidden_layer_sizes=self.hidden_layer_sizes, activation=self.activation,
                                   solver=self.solver, alpha=self.alpha, batch_size=self.batch_size,
                                   learning_rate_init=self.learning_rate_init, max_iter=self.max_iter, shuffle=True,
                                   random_state=self.seed, early_stopping=False)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore", ConvergenceWarning)  # a fixed epoch budget by design
            warnings.filterwarnings("ignore", message="Got `batch_size`")  # small splits clip the batch
            self._model.fit(X, Y)
        return self

    def predict(self, x) -> np.ndarray:
        if self._model is None:
            raise RuntimeError("RecentHistoryMLP is not fitted")
        return np.asarray(self._model.predict(self._x(x)), dtype=np.float64).reshape(-1, self.output_dim)


class NumpyCausalTCN:
    """Causal Conv1D (kernel index 0 = oldest lag, K-1 = current step) + tanh + linear head, float64."""

    _PARAMETERS = ("kernel", "conv_bias", "head_weight", "head_bias")
    _INT_CONFIG = ("input_dim", "output_dim", "kernel_size", "hidden_channels", "epochs", "batch_size", "seed")
    _FLOAT_CONFIG = ("learning_rate", "l2", "beta1", "beta2", "epsilon")

    def __init__(self, input_dim: int, output_dim: int, *, kernel_size: int = 3, hidden_channels: int = 8,
                 epochs: int = 40, batch_size: int = 256, learning_rate: float = 5e-3, l2: float = 1e-4,
                 beta1: float = 0.9, beta2: float = 0.999, epsilon: float = 1e-8, seed: int = 20260731):
        if min(input_dim, output_dim, kernel_size, hidden_channels, epochs, batch_size) <= 0:
            raise ValueError("TCN dimensions and training counts must be positive")
        self.input_dim, self.output_dim = int(input_dim), int(output_dim)
        self.kernel_size, self.hidden_channels = int(kernel_size), int(hidden_channels)
        self.epochs, self.batch_size, self.seed = int(epochs), int(batch_size), int(seed)
        self.learning_rate, self.l2 = float(learning_rate), float(l2)
        self.beta1, self.beta2, self.epsilon = float(beta1), float(beta2), float(epsilon)
        rng = np.random.default_rng(self.seed)
        k_lim = np.sqrt(6.0 / (self.kernel_size * self.input_dim + self.hidden_channels))
        h_lim = np.sqrt(6.0 / (2 * self.hidden_channels + self.output_dim))
        self.kernel = rng.uniform(-k_lim, k_lim, size=(self.kernel_size, self.input_dim, self.hidden_channels))
        self.conv_bias = np.zeros(self.hidden_channels)
        self.head_weight = rng.uniform(-h_lim, h_lim, size=(2 * self.hidden_channels, self.output_dim))
        self.head_bias = np.zeros(self.output_dim)

    @property
    def representation_dim(self) -> int:
        return 2 * self.hidden_channels

    def _check(self, x) -> np.ndarray:
        v = np.asarray(x, dtype=np.float64)
        if v.ndim != 3 or v.shape[1] == 0 or v.shape[2] != self.input_dim:
            raise ValueError("TCN input must have shape [batch, time, input_dim]")
        if not np.isfinite(v).all():
            raise ValueError("TCN input contains NaN/Inf")
        return v

    def _forward(self, x):
        v = self._check(x)
        B, T, _ = v.shape
        K = self.kernel_size
        pre = np.broadcast_to(self.conv_bias, (B, T, self.hidden_channels)).copy()
        for k in range(K):  # tap k sees step t - (K-1-k)
            lag = K - 1 - k
            if lag < T:
                pre[:, lag:] += v[:, :T - lag] @ self.kernel[k]
        h = np.tanh(pre)
        rep = np.concatenate((h[:, -1], h.mean(axis=1)), axis=1)
        return rep @ self.head_weight + self.head_bias, h, rep

    def temporal_hidden(self, x) -> np.ndarray:
        return self._forward(x)[1]

    def predict(self, x) -> np.ndarray:
        return self._forward(x)[0]

    def _penalty(self) -> float:
        return self.l2 * float(np.sum(self.kernel ** 2) + np.sum(self.head_weight ** 2))

    def loss(self, x, y) -> float:
        p = self.predict(x)
        t = np.asarray(y, dtype=np.float64)
        if t.shape != p.shape:
            raise ValueError("TCN target shape mismatch")
        return float(np.mean((p - t) ** 2)) + self._penalty()

    def loss_and_gradients(self, x, y):
        v = self._check(x)
        t = np.asarray(y, dtype=np.float64)
        p, h, rep = self._forward(v)
        if t.shape != p.shape:
            raise ValueError("TCN target shape mismatch")
        B, T, _ = v.shape
        H, K = self.hidden_channels, self.kernel_size
        err = p - t
        dp = (2.0 / err.size) * err
        g_hw = rep.T @ dp + 2.0 * self.l2 * self.head_weight
        g_hb = dp.sum(axis=0)
        drep = dp @ self.head_weight.T
        dh = np.repeat(drep[:, None, H:] / T, T, axis=1)
        dh[:, -1] += drep[:, :H]
        dpre = dh * (1.0 - h ** 2)
        g_k = np.zeros_like(self.kernel)
        for k in range(K):
            lag = K - 1 - k
            if lag < T:
                g_k[k] = v[:, :T - lag].reshape(-1, self.input_dim).T @ dpre[:, lag:].reshape(-1, H)
        g_k += 2.0 * self.l2 * self.kernel
        return float(np.mean(err ** 2)) + self._penalty(), {"kernel": g_k, "conv_bias": dpre.sum(axis=(0, 1)),
                                                           "head_weight": g_hw, "head_bias": g_hb}

    def fit(self, x, y) -> np.ndarray:
        """Adam over shuffled mini-batches; returns the full-data loss after each epoch."""
        v = self._check(x)
        t = np.asarray(y, dtype=np.float64)
        if t.shape != (len(v), self.output_dim):
            raise ValueError("TCN target shape mismatch")
        m1 = {k: np.zeros_like(getattr(self, k)) for k in self._PARAMETERS}
        m2 = {k: np.zeros_like(getattr(self, k)) for k in self._PARAMETERS}
        rng = np.random.default_rng(self.seed)
        step = 0
        hist = np.empty(self.epochs)
        for e in range(self.epochs):
            perm = rng.permutation(len(v))
            for s in range(0, len(v), self.batch_size):
                idx = perm[s:s + self.batch_size]
                _, g = self.loss_and_gradients(v[idx], t[idx])
                step += 1
                for k in self._PARAMETERS:
                    m1[k] = self.beta1 * m1[k] + (1.0 - self.beta1) * g[k]
                    m2[k] = self.beta2 * m2[k] + (1.0 - self.beta2) * g[k] ** 2
                    getattr(self, k)[...] -= (self.learning_rate * (m1[k] / (1.0 - self.beta1 ** step))
                                              / (np.sqrt(m2[k] / (1.0 - self.beta2 ** step)) + self.epsilon))
            hist[e] = self.loss(v, t)
        return hist

    def state_dict(self) -> dict[str, np.ndarray]:
        return {k: getattr(self, k).copy() for k in self._PARAMETERS}

    def load_state_dict(self, state: Mapping[str, np.ndarray]) -> None:
        if set(state) != set(self._PARAMETERS):
            raise ValueError(f"TCN state must contain exactly {self._PARAMETERS}")
        for k in self._PARAMETERS:
            a = np.asarray(state[k], dtype=np.float64)
            if a.shape != getattr(self, k).shape or not np.isfinite(a).all():
                raise ValueError(f"invalid TCN state for {k}")
            setattr(self, k, a.copy())

    def save(self, path: str | Path) -> None:
        arrays = self.state_dict()
        arrays.update({f"config_{k}": np.asarray([getattr(self, k)]) for k in self._INT_CONFIG + self._FLOAT_CONFIG})
        np.savez_compressed(path, **arrays)

    @classmethod
    def load(cls, path: str | Path) -> "NumpyCausalTCN":
        with np.load(path, allow_pickle=False) as v:
            cfg = {k: int(v[f"config_{k}"][0]) for k in cls._INT_CONFIG}
            cfg.update({k: float(v[f"config_{k}"][0]) for k in cls._FLOAT_CONFIG})
            m = cls(**cfg)
            m.load_state_dict({k: v[k] for k in cls._PARAMETERS})
        return m


class HistoryPredictorSuite:
    """The six point methods, fit on the fit split only."""

    def __init__(self, recent_steps: int, target_dim: int, seed: int = 20260731):
        self.recent_steps, self.target_dim, self.seed = int(recent_steps), int(target_dim), int(seed)
        self.moment = RidgeMultiOutput(alpha=10.0)
        self.mlp = RecentHistoryMLP(self.recent_steps * self.target_dim, self.target_dim, seed=self.seed)
        self.tcn = NumpyCausalTCN(self.target_dim, self.target_dim, seed=self.seed)
        self.long_term_mean = self.input_mean = self.input_scale = self.target_mean = self.target_scale = None

    def fit(self, moment_features, recent_history, targets) -> "HistoryPredictorSuite":
        from .data import fit_standardizers
        r, y = np.asarray(recent_history, dtype=np.float64), np.asarray(targets, dtype=np.float64)
        if r.shape[1:] != (self.recent_steps, self.target_dim) or y.shape != (len(r), self.target_dim):
            raise ValueError("suite training shapes do not match configuration")
        st = fit_standardizers(r, y)
        self.long_term_mean = y.mean(axis=0)
        self.input_mean, self.input_scale, self.target_mean, self.target_scale = (
            st.input_mean, st.input_scale, st.target_mean, st.target_scale)
        rn, yn = st.transform_inputs(r), st.transform_targets(y)
        self.moment.fit(moment_features, y)
        self.mlp.fit(rn, yn)
        self.tcn.fit(rn, yn)
        return self

    def predict(self, moment_features, recent_history, previous_targets, ewma_targets) -> dict[str, np.ndarray]:
        if self.long_term_mean is None:
            raise RuntimeError("HistoryPredictorSuite is not fitted")
        rn = (np.asarray(recent_history, dtype=np.float64) - self.input_mean) / self.input_scale
        back = lambda z: z * self.target_scale + self.target_mean  # noqa: E731
        return {"long_term_mean": np.tile(self.long_term_mean, (len(rn), 1)),
                "previous_value": np.asarray(previous_targets, dtype=np.float64).copy(),
                "ewma": np.asarray(ewma_targets, dtype=np.float64).copy(),
                "moment_only": self.moment.predict(moment_features),
                "recent_history_mlp": back(self.mlp.predict(rn)), "causal_tcn": back(self.tcn.predict(rn))}
