"""Fused producers of the input slicing (RMSNorm, SwiGLU) against the torch transform + slicing."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SLICES = [1, 1, 2, 2, 2]


def _engine(device, noisy=False):
    import memintelli_flash_b200 as M
    return M.DPETensor(device=device, HGS=1e-5, LGS=1e-8, write_variation=0.0, rate_stuck_HGS=0.0,
                       rate_stuck_LGS=0.0, read_variation=0.05 if noisy else 0.0, vnoise=0.0, rdac=4, g_level=4,
                       radc=4096)


def _input(device, gran=(1, 128)):
    import memintelli_flash_b200 as M
    return M.SlicedData(torch.tensor(SLICES), is_weight=False, paral_size=(1, 32), quant_gran=gran, device=device,
                        inference=False)


def _codes(sd):
    return sd._buf["packed"].cpu().numpy().astype(np.int64)


def _signed(c):
    return np.where(c >= 128, c - 256, c)


@pytest.mark.parametrize("shape", [(3, 37, 256), (512, 1024), (2, 64, 250)])
def test_rmsnorm_slicing(shape, cuda):
    """Codes of the fused RMSNorm slicing equal slicing x * rsqrt(mean(x^2) + eps) * w, up to one
    quantisation step on values the reordered sum of squares moves across a rounding boundary.
    K = 250 is not a multiple of 4 and takes the torch fallback, which must match exactly."""
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(*shape, device=cuda, generator=g) * 3.0
    w = torch.rand(shape[-1], device=cuda, generator=g) + 0.5
    eng = _engine(cuda)
    fused, ref = _input(cuda), _input(cuda)
    eng.slice_rmsnorm_input(fused, x, w, 1e-6)
    ref.slice_data_imp(eng, x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w)
    a, b = _signed(_codes(fused)), _signed(_codes(ref))
    assert fused.shape == ref.shape
    if shape[-1] % 4:
        assert np.array_equal(a, b)
        return
    assert np.abs(a - b).max() <= 1
    assert np.mean(a != b) <= 1e-3
    bm_f, bm_r = fused._buf["block_max"].cpu().numpy(), ref._buf["block_max"].cpu().numpy()
    assert np.allclose(bm_f, bm_r, rtol=1e-6, atol=0)


@pytest.mark.parametrize("shape,width", [((4, 33, 512), 256), ((300, 768), 384)])
def test_swiglu_slicing(shape, width, cuda):
    """Codes of the fused SwiGLU slicing equal slicing silu(gate) * up computed by torch."""
    g = torch.Generator(device=cuda).manual_seed(5)
    gu = torch.randn(*shape, device=cuda, generator=g) * 2.0
    eng = _engine(cuda)
    fused, ref = _input(cuda), _input(cuda)
    eng.slice_swiglu_input(fused, gu, width)
    ref.slice_data_imp(eng, torch.nn.functional.silu(gu[..., :width]) * gu[..., width:2 * width])
    a, b = _signed(_codes(fused)), _signed(_codes(ref))
    assert fused.shape == ref.shape
    assert np.abs(a - b).max() <= 1
    assert np.mean(a != b) <= 1e-4


def test_fused_input_feeds_mvm(cuda):
    """A fused-sliced input runs through the MVM like an ordinary one, noise-free and with read noise
    (FP16 planes straight from the slicing), and matches the unfused result."""
    import memintelli_flash_b200 as M
    g = torch.Generator(device=cuda).manual_seed(9)
    x = torch.randn(256, 512, device=cuda, generator=g)
    wn = torch.rand(512, device=cuda, generator=g) + 0.5
    w = torch.randn(512, 384, device=cuda, generator=g)
    for noisy in (False, True):
        eng = _engine(cuda, noisy)
        ws = M.SlicedData(torch.tensor(SLICES), is_weight=True, paral_size=(32, 32), quant_gran=(128, 128),
                          device=cuda, inference=True)
        ws.slice_data_imp(eng, w)
        fused, ref = _input(cuda), _input(cuda)
        eng.slice_rmsnorm_input(fused, x, wn, 1e-6)
        ref.slice_data_imp(eng, x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * wn)
        if noisy:
            assert fused._buf["planes"].dtype == torch.float16     # no E4M3 -> FP16 pass
            torch.manual_seed(0)
        yf = eng(fused, ws)
        if noisy:
            torch.manual_seed(0)                                    # same read-noise draw
        yr = eng(ref, ws)
        torch.cuda.synchronize()
        rel = float((yf - yr).norm() / yr.norm())
        assert rel <= 2e-3, rel        # a few codes differ by one step (reordered sum of squares)


@pytest.mark.parametrize("hq,hk,d", [(16, 8, 128), (4, 4, 64)])
def test_qk_norm_rope_bf16(hq, hk, d, cuda):
    """mib_qk_norm_rope_bf16 equals rope(rms_norm(q) * q_norm), rope(rms_norm(k) * k_norm) and v cast to
    bf16, computed in fp32 by torch (one bf16 rounding step at most, from the reordered sum of squares)."""
    from memintelli_flash_b200 import _native as N
    from memintelli_flash_b200.qwen3_prefill import apply_rope, rms_norm, rope_cache
    B, T = 2, 96
    g = torch.Generator(device=cuda).manual_seed(13)
    qkv = torch.randn(B, T, (hq + 2 * hk) * d, device=cuda, generator=g)
    qn = torch.rand(d, device=cuda, generator=g) + 0.5
    kn = torch.rand(d, device=cuda, generator=g) + 0.5
    cos, sin = rope_cache(T, d, 1e6, cuda)
    q, k, v = (torch.empty(B, T, n, d, dtype=torch.bfloat16, device=cuda) for n in (hq, hk, hk))
    N.call("mib_qk_norm_rope_bf16", N.ptr(qkv), B * T, qkv.stride(-2), T, hq, hk, d, N.ptr(qn), N.ptr(kn), 1e-6,
           N.ptr(cos), N.ptr(sin), N.ptr(q), N.ptr(k), N.ptr(v), N.stream_ptr(cuda))
    rq = apply_rope(rms_norm(qkv[..., :hq * d].reshape(B, T, hq, d), qn, 1e-6), cos[:, None], sin[:, None])
    rk = apply_rope(rms_norm(qkv[..., hq * d:(hq + hk) * d].reshape(B, T, hk, d), kn, 1e-6), cos[:, None],
                    sin[:, None])
    rv = qkv[..., (hq + hk) * d:].reshape(B, T, hk, d)
    assert torch.equal(v, rv.bfloat16())
    for got, want in ((q, rq), (k, rk)):
        w16 = want.bfloat16()
        # one bf16 step, or 1e-4 absolute where rope's x*cos + rot*sin cancels to a value near zero (the
        # normalised values are O(1), so fp32 differences of ~1e-7 there exceed a step of the result)
        step = (w16.float().abs() * 2.0 ** -7).clamp_min(1e-4)
        assert ((got.float() - w16.float()).abs() <= step).all()
        assert (got != w16).float().mean().item() <= 1e-2


def test_row_logsumexp_matches_torch(cuda):
    """mib_row_logsumexp (the Qwen3 driver's loss pass) against torch's fp32 logsumexp and gather, on a full
    vocabulary row block and a shard of it with targets outside the shard."""
    from memintelli_flash_b200 import _native as N
    g = torch.Generator(device=cuda).manual_seed(4)
    x = torch.randn(300, 151936, generator=g, device=cuda) * 3.0
    t = torch.randint(0, 151936, (300,), generator=g, device=cuda)
    for lo, hi in ((0, 151936), (40960, 60000)):
        blk = x[:, lo:hi]
        m, s, tg = (torch.empty(300, device=cuda) for _ in range(3))
        N.call("mib_row_logsumexp", N.ptr(blk), 300, hi - lo, blk.stride(0), N.ptr(t), lo, N.ptr(m), N.ptr(s),
               N.ptr(tg), N.stream_ptr(cuda))
        torch.cuda.synchronize()
        lse = torch.log(s) + m
        ref = torch.logsumexp(blk.double(), dim=-1)
        assert torch.allclose(lse.double(), ref, rtol=0, atol=2e-5)
        assert torch.equal(m, blk.max(dim=-1).values)
        inside = (t >= lo) & (t < hi)
        want = torch.where(inside, blk.gather(1, (t - lo).clamp(0, hi - lo - 1)[:, None])[:, 0], torch.zeros_like(m))
        assert torch.equal(tg, want)
