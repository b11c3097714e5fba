"""The q / k RMSNorm + RoPE of the LM forward on the GPU: the RoPE table
(ovb_rope_table), the unfused fp16 kernel (ovb_qk_norm_rope_f16) and the
q|k|v GEMM with it fused into its epilogue (ovb_linear_h_qk_rope).

* The table against cos / sin in float64 of the same fp32 angles
  (qk_norm_rope_f32's table, cpp/src/backend/cpu/ops_cpu.cpp:945-986).
* The unfused kernel against a float64 restatement of qk_norm_rope_f32
  (ops_cpu.cpp:945-1013) on the same table, to the fp16 rounding of the
  outputs.
* The fused GEMM against the unfused sequence (ovb_linear_h_sliced into fp32
  q / k / v, then ovb_qk_norm_rope_f16): bit for bit, for the LM's shape and
  for head layouts whose tiles mix q, k and v heads or end on a single head,
  over ragged row counts.
* Both against a float32 restatement of the kernels' rounding sequence (the
  sum of squares in the device's warp-tree order, then every product and sum
  rounded to nearest, as numpy's float32 arithmetic does): bit for bit.  A
  fused multiply-add anywhere in the device arithmetic shows up here.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import ovnative_b200 as ovb

pytestmark = pytest.mark.gpu

EPS = 1e-6
THETA = 1e6


def inv_freq(theta=THETA):
    return np.array([np.float32(theta ** (-2.0 * i / 128.0)) for i in range(64)], np.float32)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def cos_sin(tab):
    """[rows, 64, 2] (cos, sin) per angle from the table's groups of two
    angles (cos, cos, sin, sin)."""
    t = np.asarray(tab).reshape(-1, 32, 2, 2)
    return np.stack([t[:, :, 0, :].reshape(-1, 64), t[:, :, 1, :].reshape(-1, 64)], -1)


def test_rope_table_matches_cos_sin_of_the_fp32_angles(cuda):
    rng = np.random.default_rng(1)
    pos = rng.integers(0, 4096, size=777).astype(np.int64)
    tab = cos_sin(host(ovb.rope_table(torch.from_numpy(pos).to(cuda), THETA)))
    ang = (pos.astype(np.float32)[:, None] * inv_freq()[None, :]).astype(np.float32)
    np.testing.assert_allclose(tab[..., 0], np.cos(ang.astype(np.float64)), rtol=0, atol=2e-6)
    np.testing.assert_allclose(tab[..., 1], np.sin(ang.astype(np.float64)), rtol=0, atol=2e-6)


def norm_rope_ref(x, w, tab):
    """qk_norm_rope_f32 on [rows, heads, 128] in float64 with the table's
    cos / sin."""
    x = x.astype(np.float64)
    s = 1.0 / np.sqrt((x * x).sum(-1, keepdims=True) / 128.0 + EPS)
    a = x[..., :64] * s * w[:64]
    b = x[..., 64:] * s * w[64:]
    c = tab[:, None, :, 0].astype(np.float64)
    sn = tab[:, None, :, 1].astype(np.float64)
    return np.concatenate([a * c - b * sn, b * c + a * sn], -1)


def test_unfused_kernel_against_the_reference_formula(cuda):
    rng = np.random.default_rng(2)
    rows, H, KV = 301, 16, 8
    q = rng.standard_normal((rows, H * 128)).astype(np.float32) * 3
    k = rng.standard_normal((rows, KV * 128)).astype(np.float32)
    v = rng.standard_normal((rows, KV * 128)).astype(np.float32)
    qw = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kw = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    pos = np.arange(rows, dtype=np.int64)
    d = lambda a: torch.from_numpy(a).to(cuda)  # noqa: E731
    tab = ovb.rope_table(d(pos), THETA)
    q16, k16, v16 = ovb.qk_norm_rope_f16(d(q), d(k), d(v), d(qw), d(kw), EPS, tab)
    tabh = cos_sin(host(tab))
    for got, x, w, n in ((q16, q, qw, H), (k16, k, kw, KV)):
        want = norm_rope_ref(x.reshape(rows, n, 128), w, tabh).reshape(rows, n * 128)
        g = host(got).astype(np.float64)
        np.testing.assert_allclose(g, want, rtol=1e-3, atol=1e-3 * np.abs(want).max())
    np.testing.assert_array_equal(host(v16), v.astype(np.float16))
    assert ovb.device_status() == 0


def qkv_weight(rng, H, KV, K):
    parts = []
    for n in (H * 128, KV * 128, KV * 128):
        W = rng.integers(-127, 128, size=(n, K), dtype=np.int8)
        sc = (np.abs(rng.standard_normal(n)) * 0.02 / 127).astype(np.float32)
        parts.append(ovb.Weight.from_nk(W, sc, f16=True))
    w = ovb.Weight.concat(parts)
    for p in parts:
        p.close()
    return w


# pair 0: single-CTA 128 x 256 tiles; pair 1: the persistent cta_group::2
# kernel (256 x 256 per 2-CTA cluster; 3000 rows give each cluster several
# tiles, 300 rows a peer CTA without rows).
@pytest.mark.parametrize("pair", [0, 1])
@pytest.mark.parametrize("H,KV,K", [(16, 8, 1024), (2, 1, 256), (3, 1, 320), (4, 2, 64)])
@pytest.mark.parametrize("M", [1, 77, 128, 300, 1000, 3000])
def test_fused_qkv_gemm_equals_the_unfused_sequence(cuda, monkeypatch, pair, H, KV, K, M):
    monkeypatch.setenv("OVB_GEMM_TILE_N", "256")
    monkeypatch.setenv("OVB_GEMM_PAIR", str(pair))
    rng = np.random.default_rng(M * 100 + H)
    w = qkv_weight(rng, H, KV, K)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    x = d(rng.standard_normal((M, K)).astype(np.float32))
    gain = d(np.ones(K, np.float32))
    a16, _ = ovb.rmsnorm_quantize_f32(x, gain, EPS, f16=True)
    qw = d(rng.uniform(0.5, 1.5, 128).astype(np.float32))
    kw = d(rng.uniform(0.5, 1.5, 128).astype(np.float32))
    pos = d(rng.permutation(max(M, 2048))[:M].astype(np.int64))
    tab = ovb.rope_table(pos, THETA)
    q = torch.empty((M, H * 128), device=cuda)
    k = torch.empty((M, KV * 128), device=cuda)
    v = torch.empty((M, KV * 128), device=cuda)
    ovb.linear_h_sliced(a16, w, [q, k, v])
    want = ovb.qk_norm_rope_f16(q, k, v, qw, kw, EPS, tab)
    got = ovb.linear_h_qk_rope(a16, w, H, KV, qw, kw, EPS, tab)
    for g, e in zip(got, want):
        np.testing.assert_array_equal(host(g).view(np.uint16), host(e).view(np.uint16))
    assert ovb.device_status() == 0
    w.close()


def norm_rope_f32(x, w, cos, sin):
    """The kernels' rounding sequence in float32 on x [rows, heads, 128]: lane
    l's partial sum (x_l^2 + x_{l+32}^2) + (x_{l+64}^2 + x_{l+96}^2), the warp
    tree over distances 16, 8, 4, 2, 1, scale = 1 / sqrt(sum / 128 + eps),
    a = (x_i scale) w_i, b = (x_{i+64} scale) w_{i+64}, a cos - b sin and
    b cos + a sin, each operation rounded to nearest; fp16 round to nearest
    even."""
    f = np.float32
    x = x.astype(f)
    sq = x * x
    t = (sq[..., 0:32] + sq[..., 32:64]) + (sq[..., 64:96] + sq[..., 96:128])
    for o in (16, 8, 4, 2, 1):
        t = t[..., :o] + t[..., o:2 * o]
    scale = (f(1) / np.sqrt(t[..., 0] / f(128) + f(EPS))).astype(f)[..., None]
    a = (x[..., :64] * scale) * w[:64]
    b = (x[..., 64:] * scale) * w[64:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([a * c - b * s, b * c + a * s], -1).astype(np.float16)


@pytest.mark.parametrize("M", [77, 3000])
def test_fused_and_unfused_equal_the_float32_rounding_sequence(cuda, M):
    H, KV, K = 16, 8, 1024
    rng = np.random.default_rng(M + 17)
    w = qkv_weight(rng, H, KV, K)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    x = d(rng.standard_normal((M, K)).astype(np.float32))
    a16, _ = ovb.rmsnorm_quantize_f32(x, d(np.ones(K, np.float32)), EPS, f16=True)
    qw_h = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    kw_h = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    tab = ovb.rope_table(d(rng.permutation(4096)[:M].astype(np.int64)), THETA)
    q = torch.empty((M, H * 128), device=cuda)
    k = torch.empty((M, KV * 128), device=cuda)
    v = torch.empty((M, KV * 128), device=cuda)
    ovb.linear_h_sliced(a16, w, [q, k, v])
    unfused = ovb.qk_norm_rope_f16(q, k, v, d(qw_h), d(kw_h), EPS, tab)
    fused = ovb.linear_h_qk_rope(a16, w, H, KV, d(qw_h), d(kw_h), EPS, tab)
    cs = cos_sin(host(tab))
    for i, (src, wt, n) in enumerate(((q, qw_h, H), (k, kw_h, KV))):
        want = norm_rope_f32(host(src).reshape(M, n, 128), wt, cs[..., 0], cs[..., 1])
        want = want.reshape(M, n * 128).view(np.uint16)
        np.testing.assert_array_equal(host(unfused[i]).view(np.uint16), want)
        np.testing.assert_array_equal(host(fused[i]).view(np.uint16), want)
    np.testing.assert_array_equal(host(fused[2]), host(v).astype(np.float16))
    assert ovb.device_status() == 0
    w.close()


def test_fused_qkv_gemm_flags_fp16_overflow(cuda):
    """A v value beyond the fp16 range sets status bit 16 (q and k are
    normalised, so only v can leave the range)."""
    rng = np.random.default_rng(7)
    H, KV, K, M = 2, 1, 64, 40
    parts = []
    for n in (H * 128, KV * 128, KV * 128):
        W = rng.integers(-127, 128, size=(n, K), dtype=np.int8)
        parts.append(ovb.Weight.from_nk(W, np.full(n, 100.0, np.float32), f16=True))
    w = ovb.Weight.concat(parts)
    a16, _ = ovb.rmsnorm_quantize_f32(torch.full((M, K), 8.0, device=cuda),
                                      torch.full((K,), 100.0, device=cuda), EPS, f16=True)
    one = torch.ones(128, device=cuda)
    tab = ovb.rope_table(torch.arange(M, device=cuda, dtype=torch.int64), THETA)
    ovb.linear_h_qk_rope(a16, w, H, KV, one, one, EPS, tab)
    assert ovb.device_status() & 16
    for p in (*parts, w):
        p.close()


def test_table_shape_and_type_are_checked_before_the_device(cuda):
    """A RoPE table of the wrong type or too few rows is refused on the host
    (the kernels read 64 (cos, sin) pairs for every row)."""
    rng = np.random.default_rng(9)
    M, H, KV, K = 300, 2, 1, 64
    w = qkv_weight(rng, H, KV, K)
    a16 = torch.zeros((M, K), dtype=torch.float16, device=cuda)
    one = torch.ones(128, device=cuda)
    pos = torch.arange(M, device=cuda, dtype=torch.int64)
    with pytest.raises(ValueError, match="table"):
        ovb.linear_h_qk_rope(a16, w, H, KV, one, one, EPS, pos)
    short = ovb.rope_table(pos[: M // 2], THETA)
    with pytest.raises(ValueError, match="table"):
        ovb.linear_h_qk_rope(a16, w, H, KV, one, one, EPS, short)
    q = torch.zeros((M, H * 128), device=cuda)
    kv = torch.zeros((M, KV * 128), device=cuda)
    with pytest.raises(ValueError, match="table"):
        ovb.qk_norm_rope_f16(q, kv, kv, one, one, EPS, short)
    w.close()
