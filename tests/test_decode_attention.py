"""Decode attention against a static KV cache (``ferrite_attn_decode``): the
reference's decode-step ``_write_cache`` + ``_cache_attention``
(src/ferrite/serving/engine.py:89-104), fused into one kernel.

CPU: the oracle's ``decode_reference`` agrees with the causal reference attention
row it must equal, reproduces the committed golden fixture, and the C ABI rejects
bad arguments before touching a device.
GPU (``-m gpu``): the kernel against the oracle and the fixture (outputs within
the bf16 tolerance of the attention tests, 2e-2 max-abs; f32 within 2e-5), the
cache rows it writes bit-exact, every other row untouched, a position outside the
cache a NaN row with no write, and a long cache against the torch f32 reference.
"""

import os

import numpy as np
import pytest
import torch

from helpers import BF16, load_arrays, normal, to_torch
from oracle import attention as oa

from ferrite import _native as nat

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "decode_bf16_4x2x160x64.npz")


# --------------------------------------------------------------------------- CPU


def test_oracle_decode_equals_causal_reference_row():
    rng = np.random.default_rng(0)
    b, h, s, d = 2, 3, 48, 32
    q, k, v = (normal(rng, (b, h, s, d), np.float32) for _ in range(3))
    junk = normal(rng, (b, h, 16, d), np.float32, std=5.0)  # rows after pos must not matter
    for p in (0, 1, 17, s - 1):
        kc = np.concatenate([k, junk], axis=2)
        vc = np.concatenate([v, junk], axis=2)
        kc[:, :, p + 1 : s] = 7.0
        vc[:, :, p + 1 : s] = -7.0
        o, _, _ = oa.decode_reference(q[:, :, p], kc, vc, np.full(b, p), 1.0 / np.sqrt(d))
        ref = oa.reference_fwd(q[:, :, : p + 1], k[:, :, : p + 1], v[:, :, : p + 1], causal=True)[:, :, p]
        np.testing.assert_allclose(o, ref, rtol=1e-5, atol=1e-6)


def test_oracle_decode_writes_the_new_rows():
    rng = np.random.default_rng(1)
    b, h, L, d = 3, 2, 20, 8
    q, kn, vn = (normal(rng, (b, h, d), BF16) for _ in range(3))
    kc, vc = (normal(rng, (b, h, L, d), BF16) for _ in range(2))
    pos = np.array([0, 9, L - 1])
    o, kc2, vc2 = oa.decode_reference(q, kc, vc, pos, 0.3, kn, vn)
    for bi, p in enumerate(pos):
        assert np.array_equal(kc2[bi, :, p], kn[bi]) and np.array_equal(vc2[bi, :, p], vn[bi])
        keep = np.arange(L) != p
        assert np.array_equal(kc2[bi, :, keep], kc[bi, :, keep])
    # the new row takes part: attending to the written cache without k_new gives the same output
    o2, _, _ = oa.decode_reference(q, kc2, vc2, pos, 0.3)
    assert np.array_equal(o.view(np.uint16), o2.view(np.uint16))


def test_decode_golden_fixture_reproduces():
    g = load_arrays(GOLDEN)
    o, _, _ = oa.decode_reference(g["q"], g["k_cache"], g["v_cache"], g["pos"], 0.125, g["k_new"], g["v_new"])
    assert np.array_equal(o.view(np.uint16), g["o"].view(np.uint16))


def test_decode_capi_validation_without_a_gpu():
    lib = nat.lib()
    f = lib.ferrite_attn_decode
    # b, h, max_len, d, ld_new, scale, dtype
    assert f(None, 16, 16, 16, 16, 16, 16, 16, 2, 4, 128, 48, 4 * 48, 0.1, nat.BF16) == nat.BAD_SHAPE
    assert "head_dim 48" in nat.last_error()
    assert f(None, 16, 16, 16, 16, 16, 16, 16, 2, 4, 128, 256, 4 * 256, 0.1, nat.F32) == nat.BAD_SHAPE
    assert f(None, 16, 16, None, 16, 16, 16, 16, 2, 4, 128, 64, 4 * 64, 0.1, nat.BF16) == nat.BAD_SHAPE
    assert "both" in nat.last_error()
    assert f(None, 16, 16, 16, 16, 16, 16, 16, 2, 4, 128, 64, 64, 0.1, nat.BF16) == nat.BAD_SHAPE  # ld_new < h*d
    assert f(None, 8, 16, 16, 16, 16, 16, 16, 2, 4, 128, 64, 4 * 64, 0.1, nat.BF16) == nat.BAD_ALIGNMENT
    assert f(None, 16, 16, 16, 16, 16, 16, 16, 2, 4, 128, 64, 4 * 64 + 4, 0.1, nat.BF16) == nat.BAD_ALIGNMENT
    assert f(None, 16, 16, 16, 16, 16, 16, 16, 2, 4, 128, 64, 4 * 64, 0.1, 9) == nat.UNSUPPORTED_DTYPE
    assert f(None, None, None, None, None, None, None, None, 0, 4, 128, 64, 4 * 64, 0.1, nat.BF16) == nat.OK


def test_decode_python_api_refuses_cpu_tensors():
    from ferrite.kernels.decode_attention import decode_attention

    q = torch.zeros(1, 1, 64, dtype=torch.bfloat16)
    kc = torch.zeros(1, 1, 8, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        decode_attention(q, kc, kc.clone(), torch.zeros(1, dtype=torch.long))


def _cluster(bh, max_len, d=64, dtype=None, slots=296):
    """The cluster size the compiled rule in csrc/decode.cu picks (host-only query)."""
    return nat.lib().ferrite_attn_decode_cluster(bh, max_len, d, nat.BF16 if dtype is None else dtype, slots)


def test_cluster_rule_fills_one_wave():
    # the bench shape: 8 x 16 slices, 1024 positions, d = 64 bf16 (32 lane groups per CTA),
    # 148 SMs x 2 resident CTAs -> 2 CTAs per slice, 256 CTAs (measured best of 1/2/4/8)
    assert _cluster(128, 1024) == 2
    groups = 32  # d = 64, 16-bit: 8 lanes a row, 4 rows a warp, 8 warps
    for bh in (1, 3, 16, 37, 128, 148, 300, 4096):
        for max_len in (1, 31, 64, 512, 8192):
            c = _cluster(bh, max_len)
            assert c in (1, 2, 4, 8)
            assert c == 1 or (bh * c <= 296 and max_len // c >= groups)
            assert c == 8 or bh * 2 * c > 296 or max_len // (2 * c) < groups  # maximal
    # lane groups follow (d, dtype): d = 128 bf16 has 16 per CTA, f32 d = 128 has 8
    assert _cluster(1, 64, d=128) == 4 and _cluster(1, 64, d=128, dtype=nat.F32) == 8
    assert _cluster(0, 64) == -1 and _cluster(4, 64, d=48) == -1


def test_decode_bench_bytes_per_step():
    import bench

    # 24 layers x 8 x 16 slices at pos 1023, d = 64 bf16: the 1023 cached K and V rows plus
    # q / k_new / v_new / o and the two written rows, 128 bytes each
    per_slice = (2 * 1023 + 6) * 64 * 2
    assert bench.DecodeWorkload.step_bytes(24, 8, 16, 1023, 64) == 24 * 8 * 16 * per_slice == 806_879_232


# --------------------------------------------------------------------------- GPU


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(BF16)
    return t.numpy()


def _run(q, kc, vc, pos, scale, kn=None, vn=None):
    from ferrite.kernels.decode_attention import decode_attention

    o = decode_attention(q, kc, vc, pos, scale=scale, k_new=kn, v_new=vn)
    torch.cuda.synchronize()
    return o


@pytest.mark.gpu
def test_decode_matches_golden_fixture():
    g = load_arrays(GOLDEN)
    q, kn, vn, kc, vc = (to_torch(g[n]) for n in ("q", "k_new", "v_new", "k_cache", "v_cache"))
    pos = torch.from_numpy(g["pos"]).cuda()
    o = _run(q, kc, vc, pos, 0.125, kn, vn)
    assert (o.float() - to_torch(g["o"]).float()).abs().max().item() <= 2e-2
    kc_ref, vc_ref = to_torch(g["k_cache"]), to_torch(g["v_cache"])
    for bi, p in enumerate(g["pos"]):
        kc_ref[bi, :, p] = kn[bi]
        vc_ref[bi, :, p] = vn[bi]
    assert torch.equal(kc, kc_ref) and torch.equal(vc, vc_ref)


@pytest.mark.gpu
@pytest.mark.parametrize(
    "dtype,d,b,h,max_len",
    [
        (torch.bfloat16, 64, 8, 16, 512),
        (torch.bfloat16, 32, 3, 5, 77),
        (torch.bfloat16, 128, 2, 8, 1000),
        (torch.bfloat16, 256, 2, 2, 300),
        (torch.float16, 64, 4, 4, 129),
        (torch.float16, 128, 1, 16, 2048),
        (torch.float32, 128, 2, 1, 256),
        (torch.float32, 32, 5, 3, 64),
    ],
)
def test_decode_matches_oracle(dtype, d, b, h, max_len):
    g = torch.Generator(device="cuda").manual_seed(d * 1000 + max_len)
    kc = torch.randn(b, h, max_len, d, device="cuda", generator=g).to(dtype)
    vc = torch.randn(b, h, max_len, d, device="cuda", generator=g).to(dtype)
    qkv = torch.randn(b, 3, h, d, device="cuda", generator=g).to(dtype)  # the projection, read in place
    q, kn, vn = qkv[:, 0], qkv[:, 1], qkv[:, 2]
    pos = torch.randint(0, max_len, (b,), device="cuda", generator=g)
    pos[0] = 0
    if b > 1:
        pos[-1] = max_len - 1
    kc0, vc0 = kc.clone(), vc.clone()
    scale = 1.0 / np.sqrt(d)
    o = _run(q, kc, vc, pos, scale, kn, vn)
    o_ref, kc_ref, vc_ref = oa.decode_reference(_np(q), _np(kc0), _np(vc0), _np(pos), scale, _np(kn), _np(vn))
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    assert np.abs(_np(o).astype(np.float32) - o_ref.astype(np.float32)).max() <= tol
    assert np.array_equal(_np(kc).view(np.uint8), kc_ref.view(np.uint8))
    assert np.array_equal(_np(vc).view(np.uint8), vc_ref.view(np.uint8))


@pytest.mark.gpu
def test_decode_read_only_and_repeatable():
    """Without new rows the cache is only read; two calls give the same bits."""
    g = torch.Generator(device="cuda").manual_seed(5)
    b, h, L, d = 4, 8, 700, 64
    kc = torch.randn(b, h, L, d, device="cuda", generator=g).bfloat16()
    vc = torch.randn(b, h, L, d, device="cuda", generator=g).bfloat16()
    q = torch.randn(b, h, d, device="cuda", generator=g).bfloat16()
    pos = torch.tensor([3, 699, 350, 64], device="cuda")
    kc0, vc0 = kc.clone(), vc.clone()
    o1 = _run(q, kc, vc, pos, 0.125)
    o2 = _run(q, kc, vc, pos, 0.125)
    assert torch.equal(kc, kc0) and torch.equal(vc, vc0) and torch.equal(o1, o2)
    o_ref, _, _ = oa.decode_reference(_np(q), _np(kc0), _np(vc0), _np(pos), 0.125)
    assert np.abs(_np(o1).astype(np.float32) - o_ref.astype(np.float32)).max() <= 2e-2


@pytest.mark.gpu
def test_decode_position_outside_the_cache_gives_nan_and_no_write():
    g = torch.Generator(device="cuda").manual_seed(6)
    b, h, L, d = 3, 2, 40, 64
    kc = torch.randn(b, h, L, d, device="cuda", generator=g).bfloat16()
    vc = torch.randn(b, h, L, d, device="cuda", generator=g).bfloat16()
    q, kn, vn = (torch.randn(b, h, d, device="cuda", generator=g).bfloat16() for _ in range(3))
    pos = torch.tensor([5, L, -1], device="cuda")
    kc0, vc0 = kc.clone(), vc.clone()
    o = _run(q, kc, vc, pos, 0.125, kn, vn)
    assert torch.isnan(o[1:].float()).all() and torch.isfinite(o[0].float()).all()
    assert torch.equal(kc[1:], kc0[1:]) and torch.equal(vc[1:], vc0[1:])
    assert torch.equal(kc[0, :, 5], kn[0]) and torch.equal(vc[0, :, 5], vn[0])


@pytest.mark.gpu
def test_decode_long_cache_against_torch_f32_reference():
    from ferrite.kernels.decode_attention import decode_attention_reference

    g = torch.Generator(device="cuda").manual_seed(7)
    b, h, L, d = 8, 16, 8192, 128
    kc = torch.randn(b, h, L, d, device="cuda", generator=g).bfloat16()
    vc = torch.randn(b, h, L, d, device="cuda", generator=g).bfloat16()
    q = torch.randn(b, h, d, device="cuda", generator=g).bfloat16()
    pos = torch.randint(0, L, (b,), device="cuda", generator=g)
    pos[0] = L - 1
    o = _run(q, kc, vc, pos, None)
    ref = decode_attention_reference(q, kc, vc, pos)
    assert (o.float() - ref.float()).abs().max().item() <= 2e-2


@pytest.mark.gpu
def test_engine_decode_kernel_matches_plain_decode():
    from ferrite.model.gpt import GPTConfig, init_params
    from ferrite.serving.engine import Engine, ServeConfig

    torch.backends.cuda.matmul.allow_tf32 = False
    cfg = GPTConfig(vocab_size=256, seq_len=256, d_model=128, n_head=2, n_layer=2, d_ff=256, dtype=torch.float32)
    params = init_params(0, cfg)
    prompts = [[1, 2, 3, 4, 5, 6, 7, 8, 9, 10], [42, 7, 99]]
    outs = []
    for mode in ("pallas", "xla"):
        eng = Engine(params, cfg, ServeConfig(batch=2, max_len=256, buckets=(128,), decode_kernels=mode))
        gen, _ = eng.generate(prompts, max_new_tokens=8)
        outs.append(gen)
    np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.gpu
def test_engine_decode_graph_matches_eager_engine():
    """The captured decode step (one CUDA graph for every position) generates the same
    tokens as the eager engine, bf16 with the decode kernel at head_dim 64."""
    from ferrite.model.gpt import GPTConfig, init_params
    from ferrite.serving.engine import Engine, ServeConfig

    cfg = GPTConfig(vocab_size=512, seq_len=512, d_model=256, n_head=4, n_layer=2, d_ff=1024, linear="pallas")
    params = init_params(0, cfg)
    rng = np.random.default_rng(0)
    prompts = [list(rng.integers(0, 512, size=n)) for n in (100, 17, 128, 60)]
    outs = []
    for graphs in (True, False):
        eng = Engine(params, cfg, ServeConfig(batch=4, max_len=256, buckets=(128,), use_graphs=graphs))
        assert eng.n_compiles == 2
        gen, stats = eng.generate(prompts, max_new_tokens=12)
        assert stats["itl_ms_median"] > 0
        outs.append(gen)
    np.testing.assert_array_equal(outs[0], outs[1])
