"""Action unnormalisation (flashact_b200.postprocess): the openpi z-score and quantile maps the
reference applies on the host after readback (src/pi05/hybrid_model.py:222-228)."""
import numpy as np
import torch

from flashact_b200.postprocess import unnormalize_actions


def test_zscore_and_quantile_numpy():
    x = np.array([[0.5, -1.0, 2.0, 9.0], [1.0, 1.0, -1.0, 9.0]], dtype=np.float32)
    z = unnormalize_actions(x, {"mean": [1.0, 2.0, 3.0], "std": [2.0, 0.5, 1.0]})
    np.testing.assert_allclose(z[:, :3], x[:, :3] * (np.array([2.0, 0.5, 1.0]) + 1e-6) + [1.0, 2.0, 3.0], rtol=1e-6)
    assert (z[:, 3] == 9.0).all()  # dims without statistics pass through
    q = unnormalize_actions(x, {"q01": [0.0, -2.0, 10.0], "q99": [1.0, 2.0, 20.0]}, output_dim=3)
    assert q.shape == (2, 3)
    np.testing.assert_allclose(q[1], [1.0 + 1e-6, 2.0 + 1e-6, 10.0], rtol=1e-6)  # x = +1 -> q99, x = -1 -> q01
    np.testing.assert_allclose(q[0, 1], -2.0, rtol=1e-6)


def test_torch_matches_numpy_and_quantiles_preferred():
    x = torch.randn(3, 50, 32, generator=torch.Generator().manual_seed(0))
    stats = {"mean": np.zeros(7), "std": np.ones(7), "q01": -np.ones(7), "q99": np.ones(7) * 3}
    t = unnormalize_actions(x, stats, output_dim=7)
    n = unnormalize_actions(x.numpy(), stats, output_dim=7)
    assert isinstance(t, torch.Tensor) and t.shape == (3, 50, 7)
    np.testing.assert_allclose(t.numpy(), n, rtol=1e-6)
    np.testing.assert_allclose(n, (x.numpy()[..., :7] + 1) * 0.5 * (4 + 1e-6) - 1, rtol=1e-5, atol=1e-6)
    zs = unnormalize_actions(x, stats, use_quantiles=False)
    np.testing.assert_allclose(zs.numpy()[..., :7], x.numpy()[..., :7] * (1 + 1e-6), rtol=1e-5, atol=1e-6)
    assert torch.equal(zs[..., 7:], x[..., 7:])
