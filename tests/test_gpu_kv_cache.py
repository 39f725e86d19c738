"""The resident K/V cache (multi-step decode with K and V kept on the device):
every step matches the decode step over the same tokens computed from scratch
(the oracle, and attn_step_dense on host arrays), through the NumPy API and the
device API, with appends, truncation and the capacity limit."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL_FP32, rel_err

pytestmark = pytest.mark.gpu


def _tokens(rng, H, n, Dh):
    return (rng.standard_normal((H, n, Dh), dtype=np.float32),
            rng.standard_normal((H, n, Dh), dtype=np.float32))


@pytest.mark.parametrize("H,Dh,T0", [(4, 64, 100), (8, 128, 1), (3, 48, 257)])
def test_steps_match_from_scratch(cuda, H, Dh, T0):
    import attn_cpu

    rng = np.random.default_rng(H * 1000 + Dh + T0)
    K, V = _tokens(rng, H, T0, Dh)
    cache = attn_cpu.KVCache(H, Dh, T0 + 8)
    cache.append(K, V)
    assert len(cache) == T0
    for step in range(5):
        q = rng.standard_normal((H, Dh), dtype=np.float32)
        kn, vn = (x[:, 0] for x in _tokens(rng, H, 1, Dh))
        o = cache.step(q, kn, vn)
        K = np.concatenate([K, kn[:, None]], axis=1)
        V = np.concatenate([V, vn[:, None]], axis=1)
        assert len(cache) == T0 + step + 1
        assert rel_err(o, oracle.attn_step(q, K, V)) < TOL_FP32
        assert rel_err(o, attn_cpu.attn_step_dense(q, K, V)) < 1e-6
    # A step without a new token attends over what is there.
    q = rng.standard_normal((H, Dh), dtype=np.float32)
    assert rel_err(cache.step(q), oracle.attn_step(q, K, V)) < TOL_FP32


def test_truncate_and_refill(cuda):
    import attn_cpu

    rng = np.random.default_rng(11)
    H, Dh = 2, 32
    K, V = _tokens(rng, H, 60, Dh)
    cache = attn_cpu.KVCache(H, Dh, 64)
    cache.append(K[:, :40], V[:, :40])
    cache.append(K[:, 40:], V[:, 40:])
    cache.truncate(25)
    q = rng.standard_normal((H, Dh), dtype=np.float32)
    assert rel_err(cache.step(q), oracle.attn_step(q, K[:, :25], V[:, :25])) < TOL_FP32
    K2, V2 = _tokens(rng, H, 39, Dh)  # exactly fills the capacity again
    cache.append(K2, V2)
    assert len(cache) == 64
    Kc, Vc = np.concatenate([K[:, :25], K2], 1), np.concatenate([V[:, :25], V2], 1)
    assert rel_err(cache.step(q), oracle.attn_step(q, Kc, Vc)) < TOL_FP32


def test_errors(cuda):
    import attn_cpu

    rng = np.random.default_rng(12)
    cache = attn_cpu.KVCache(2, 16, 4)
    q = rng.standard_normal((2, 16), dtype=np.float32)
    with pytest.raises(ValueError):
        cache.step(q)  # empty
    K, V = _tokens(rng, 2, 5, 16)
    with pytest.raises(ValueError, match="capacity"):
        cache.append(K, V)
    assert len(cache) == 0  # a rejected append changes nothing
    with pytest.raises(ValueError):
        cache.append(K[:1], V[:1])  # wrong H
    with pytest.raises(ValueError):
        cache.step(q, K[:, 0])  # k_new without v_new
    with pytest.raises(ValueError):
        cache.truncate(1)  # beyond the current length
    with pytest.raises(ValueError):
        attn_cpu.KVCache(0, 16, 4)


def test_device_api_on_a_stream(cuda):
    import torch
    from attn_cpu import capi

    H, Dh, T0 = 8, 64, 200
    g = torch.Generator(device="cuda").manual_seed(13)
    K = torch.randn(H, T0, Dh, device="cuda", generator=g)
    V = torch.randn(H, T0, Dh, device="cuda", generator=g)
    s = torch.cuda.Stream()
    cache = capi.KVCacheDev(H, Dh, T0 + 4)
    with torch.cuda.stream(s):
        cache.append(K, V)
        outs, qs, news = [], [], []
        for _ in range(3):
            q = torch.randn(H, Dh, device="cuda", generator=g)
            kn = torch.randn(H, Dh, device="cuda", generator=g)
            vn = torch.randn(H, Dh, device="cuda", generator=g)
            o = torch.empty(H, Dh, device="cuda")
            cache.step(q, o, kn, vn)
            outs.append(o)
            qs.append(q)
            news.append((kn, vn))
    s.synchronize()
    capi.stream_status(s)
    Kh, Vh = K.cpu().numpy(), V.cpu().numpy()
    for o, q, (kn, vn) in zip(outs, qs, news):
        Kh = np.concatenate([Kh, kn.cpu().numpy()[:, None]], 1)
        Vh = np.concatenate([Vh, vn.cpu().numpy()[:, None]], 1)
        assert rel_err(o.cpu().numpy(), oracle.attn_step(q.cpu().numpy(), Kh, Vh)) < TOL_FP32
    assert len(cache) == T0 + 3
    cache.close()
