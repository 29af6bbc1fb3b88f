"""Action post-processing after the denoise loop: unnormalisation and the output-dimension cut.

The reference does this on the host, in numpy, after reading the action chunk back
(src/pi05/hybrid_model.py:222-228: `unnormalize_actions(raw, self.norm_stats)` from FlashRT, then
`[:, :output_dim]`). FlashRT is not part of the reference tree; the two normalisations it applies
are the published openpi ones, restated here:
  * z-score:   a = x * (std + 1e-6) + mean
  * quantile:  a = (x + 1) / 2 * (q99 - q01 + 1e-6) + q01   (x in [-1, 1] maps onto [q01, q99])
Statistics cover the first len(stats) action dims; the remaining dims pass through unchanged
(the padded dims of a 32-wide action buffer). Works on numpy arrays or torch tensors (any device).
"""
from __future__ import annotations

EPS = 1e-6


def _as(x, like):
    import numpy as np
    try:
        import torch
        if isinstance(like, torch.Tensor):
            return torch.as_tensor(np.asarray(x, dtype=np.float32), device=like.device)
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, dtype=np.float32)


def unnormalize_actions(actions, norm_stats: dict, use_quantiles: bool | None = None, output_dim: int | None = None):
    """actions [..., AD] (the chunk the engine returns) -> unnormalised actions [..., output_dim].

    norm_stats: {"mean", "std"} and/or {"q01", "q99"} per-dim sequences (length <= AD).
    use_quantiles: None = quantile statistics when present, else z-score."""
    if use_quantiles is None:
        use_quantiles = "q01" in norm_stats and "q99" in norm_stats
    keys = ("q01", "q99") if use_quantiles else ("mean", "std")
    for k in keys:
        if k not in norm_stats:
            raise KeyError(f"norm_stats lacks '{k}'")
    a, b = (_as(norm_stats[k], actions) for k in keys)
    n = a.shape[-1]
    if b.shape[-1] != n or n > actions.shape[-1]:
        raise ValueError(f"statistics of {n} / {b.shape[-1]} dims for {actions.shape[-1]}-dim actions")
    head, tail = actions[..., :n], actions[..., n:]
    if use_quantiles:
        head = (head + 1.0) * 0.5 * (b - a + EPS) + a
    else:
        head = head * (b + EPS) + a
    try:
        import torch
        out = torch.cat([head, tail], -1) if isinstance(actions, torch.Tensor) else None
    except ImportError:  # pragma: no cover
        out = None
    if out is None:
        import numpy as np
        out = np.concatenate([head, tail], -1)
    return out if output_dim is None else out[..., :output_dim]
