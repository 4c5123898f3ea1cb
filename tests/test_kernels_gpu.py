"""Kernel parity on the GPU, through the C ABI (libnpl_w8a8.so), against the
numpy oracle and the reference's golden fixtures.

Integer and byte results (int8 activations, weights, scales, int32
accumulators, fp16 epilogue outputs) must be bit-exact. Attention is fp32
arithmetic: tolerance stated per test.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import w8a8 as O

pytestmark = pytest.mark.gpu


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def K(cuda_device):
    from nanopointllm_b200 import _lib, paged_attention, runner, w8a8
    return type("K", (), dict(lib=_lib, W=w8a8, PA=paged_attention, R=runner, dev=cuda_device))


def cpu(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


# ------------------------------------------------------------ quantisation
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("rows,cols", [(8, 4096), (5, 768), (1, 16), (64, 11008), (3, 48),
                                       (300, 4096), (1001, 11008)])  # > 64 rows: 4 rows per CTA
def test_quant_rows_bit_exact(K, dtype, rows, cols):
    g = torch.Generator().manual_seed(rows * 7 + cols)
    x = torch.randn(rows, cols, generator=g) * 3
    x[:, :: max(1, cols // 40)] *= 20.0
    if rows > 1:
        x[1] = 0.0  # all-zero row: scale clamps to fp16.tiny
    x = x.to(dtype)
    q, s = K.W.dynamic_per_token_quant(x.to(K.dev))
    qo, so = O.dynamic_per_token_quant(x.numpy())
    np.testing.assert_array_equal(cpu(q), qo)
    np.testing.assert_array_equal(cpu(s), so)


def test_quant_rows_every_fp16_value(K):
    """Every finite fp16 value v with |v| <= A, quantised with the scale of a
    row whose absmax is A, for ~200 A across the fp16 range: the kernel's
    quotient (reciprocal + one FMA correction step) rounds like the IEEE fp32
    division of the reference, bit for bit."""
    allh = np.arange(1 << 16, dtype=np.uint16).view(np.float16)
    allh = allh[np.isfinite(allh)]
    amaxes = np.unique(np.concatenate([
        np.geomspace(6.2e-5, 65504, 160), [1.0, 127.0, 2.0 ** -14, 3e-5, 1e-7, 0.0],
        np.random.default_rng(0).uniform(0.01, 100, 40)]).astype(np.float16))
    width = (allh.size + 1 + 15) // 16 * 16  # every value + the row's absmax
    rows = np.zeros((amaxes.size, width), dtype=np.float16)
    for i, a in enumerate(amaxes):
        v = allh[np.abs(allh.astype(np.float32)) <= np.float32(a)]
        rows[i, :v.size] = v
        rows[i, v.size] = a  # the row's absmax is exactly a
    q, s = K.W.dynamic_per_token_quant(torch.from_numpy(rows).to(K.dev))
    qo, so = O.dynamic_per_token_quant(rows)
    np.testing.assert_array_equal(cpu(s), so)
    np.testing.assert_array_equal(cpu(q), qo)
    # fp32 inputs: sampled
    g = torch.Generator().manual_seed(5)
    x = torch.randn(64, 65536, generator=g) * torch.logspace(-6, 4, 64).reshape(-1, 1)
    q, s = K.W.dynamic_per_token_quant(x.to(K.dev))
    qo, so = O.dynamic_per_token_quant(x.numpy())
    np.testing.assert_array_equal(cpu(s), so)
    np.testing.assert_array_equal(cpu(q), qo)


def test_quant_every_fp16_value_at_every_scale(K):
    """Exhaustive: every finite fp16 value v quantised with every scale the
    per-token quantiser can produce (every fp16 value s = scale_from_absmax(A)
    for a finite fp16 absmax A: 23377 scales, 2^-14 .. 516), through npl_quant_rows_absmax:
    the kernel's quotient (the row's reciprocal + one FMA correction step)
    rounds like the IEEE fp32 division v / s of the reference, bit for bit,
    clamp included (|v| beyond 127.5 s)."""
    allh = np.arange(1 << 16, dtype=np.uint16).view(np.float16)
    allh = allh[np.isfinite(allh)]  # 63488 values, a multiple of 16
    amax = np.concatenate([[0.0], allh[allh > 0]]).astype(np.float32)
    scales = O.scale_from_absmax(amax)
    _, first = np.unique(scales, return_index=True)
    amax, scales = amax[first], scales[first]  # one absmax per distinct scale
    v = torch.from_numpy(allh).to(K.dev)
    vf = v.float()
    for c0 in range(0, amax.size, 2048):
        a = torch.from_numpy(amax[c0:c0 + 2048]).to(K.dev)
        rows = v.unsqueeze(0).expand(a.numel(), -1).contiguous()
        q, sc = K.W.quant_rows_absmax(rows, a.view(torch.int32))
        assert torch.equal(sc, torch.from_numpy(scales[c0:c0 + 2048]).to(K.dev))
        ref = torch.round(vf.unsqueeze(0) / sc.unsqueeze(1)).clamp(-127, 127).to(torch.int8)
        assert torch.equal(q, ref), f"scales {c0}..{c0 + a.numel()}"
    assert amax.size > 23000


def test_quant_golden_small(K):
    g = golden("linear_small.npz")
    for tag in ("f32", "f16"):
        x = torch.from_numpy(g[f"{tag}_x"]).to(K.dev)
        q, s = K.W.dynamic_per_token_quant(x)
        np.testing.assert_array_equal(cpu(q), g[f"{tag}_qa"])
        np.testing.assert_array_equal(cpu(s), g[f"{tag}_scale"])
        qw, sw = K.W.per_output_weight_quant(torch.from_numpy(g[f"{tag}_w"]).to(K.dev))
        np.testing.assert_array_equal(cpu(qw), g[f"{tag}_qw"])
        np.testing.assert_array_equal(cpu(sw), g[f"{tag}_ws"])


def test_rmsnorm_quant_bit_exact_and_reference_bound(K):
    g = golden("rmsnorm_quant.npz")
    x = torch.from_numpy(g["x"]).to(K.dev)
    res = torch.from_numpy(g["res"]).to(K.dev)
    w = torch.from_numpy(g["w"]).to(K.dev)
    for residual in (None, res):
        normed = torch.empty_like(x)
        q, s, summed = K.R.rmsnorm_quant(x, w, 1e-6, residual, normed_out=normed)
        qo, so, no, suo = O.rmsnorm_quant(g["x"], g["w"], 1e-6, None if residual is None else g["res"])
        np.testing.assert_array_equal(cpu(normed), no)
        np.testing.assert_array_equal(cpu(q), qo)
        np.testing.assert_array_equal(cpu(s), so)
        if residual is not None:
            np.testing.assert_array_equal(cpu(summed), g["summed"])
            ref_q = g["q_res"]
        else:
            ref_q = g["q"]
        d = np.abs(cpu(q).astype(np.int32) - ref_q.astype(np.int32))
        assert d.max() <= 1 and (d > 0).sum() <= 0.0005 * d.size


@pytest.mark.parametrize("rows,cols", [(1, 4096), (8, 4096), (64, 4096), (3, 512), (8, 11008),
                                       (301, 4096), (130, 11008), (70, 20000)])  # prefill-sized batches
def test_rmsnorm_quant_shapes(K, rows, cols):
    gen = torch.Generator().manual_seed(cols + rows)
    x = torch.randn(rows, cols, generator=gen).half()
    r = (torch.randn(rows, cols, generator=gen) * 0.1).half()
    w = (1 + 0.1 * torch.randn(cols, generator=gen)).half()
    q, s, summed = K.R.rmsnorm_quant(x.to(K.dev), w.to(K.dev), 1e-6, r.to(K.dev))
    qo, so, _, suo = O.rmsnorm_quant(x.numpy(), w.numpy(), 1e-6, r.numpy())
    np.testing.assert_array_equal(cpu(summed), suo)
    np.testing.assert_array_equal(cpu(q), qo)
    np.testing.assert_array_equal(cpu(s), so)
    if rows > 64:  # the same rows in a decode-sized batch (one row per CTA): identical bits
        q8, s8, _ = K.R.rmsnorm_quant(x[:8].to(K.dev), w.to(K.dev), 1e-6, r[:8].to(K.dev))
        assert torch.equal(q8.cpu(), q[:8].cpu()) and torch.equal(s8.cpu(), s[:8].cpu())


# ------------------------------------------------------------------ linear
def test_config1_full_size_against_reference_digest(K):
    """Config 1 at full size (8x4096 @ 12288x4096, seed 0): every quantity
    bit-exact with the reference's integer golden."""
    from nanopointllm_b200 import synthetic as S
    d = golden("config1_digest.json")
    x, w = S.config1_inputs(seed=0)
    xg, wg = x.to(K.dev), w.to(K.dev)
    qa, sa = K.W.dynamic_per_token_quant(xg)
    qw, sw = K.W.per_output_weight_quant(wg)
    assert sha(cpu(sa)) == d["sha256_act_scale_f32"]
    assert sha(cpu(qa)) == d["sha256_qact_int8"]
    assert sha(cpu(qw)) == d["sha256_qweight_int8"]
    assert sha(cpu(sw)) == d["sha256_wscale_f32"]
    out, acc = K.W.integer_linear_per_output(xg, wg)
    assert sha(cpu(acc)) == d["sha256_acc_int32"]
    assert sha(cpu(out)) == d["sha256_out_f32"]
    out16 = K.W.linear_q(qa, sa.reshape(-1), qw, sw, out_dtype=torch.float16)
    assert sha(cpu(out16)) == d["sha256_out_f16"]


@pytest.mark.parametrize("tag", ["f32", "f16"])
def test_linear_golden_small_with_bias(K, tag):
    g = golden("linear_small.npz")
    x = torch.from_numpy(g[f"{tag}_x"]).to(K.dev)
    w = torch.from_numpy(g[f"{tag}_w"]).to(K.dev)
    out, acc = K.W.integer_linear_per_output(x, w)
    np.testing.assert_array_equal(cpu(acc), g[f"{tag}_acc"])
    np.testing.assert_array_equal(cpu(out), g[f"{tag}_out"])
    out_b, _ = K.W.integer_linear_per_output(x, w, bias=torch.from_numpy(g[f"{tag}_bias"]).to(K.dev))
    np.testing.assert_array_equal(cpu(out_b), g[f"{tag}_out_bias"])


def _rand_q(gen, *shape):
    return torch.randint(-127, 128, shape, generator=gen, dtype=torch.int8)


# Prefill tiles (M > 64): 128- and 256-token tiles, two epilogue warpgroups.
# (120, 40000, 128) and (600, 12800, 256) have two waves of tiles: one wave of
# whole tiles, then stream-K over the rest; (2100, 8192, 256) has three waves
# (every tile whole), a ragged raster group of token tiles (9 = 8 + 1) and a
# ragged last token tile.
LINEAR_SHAPES = [
    (1, 384, 512), (3, 200, 768), (8, 12288, 4096), (8, 4096, 11008), (16, 1000, 512),
    (33, 640, 256), (64, 4096, 4096), (100, 512, 1024), (300, 384, 512), (8, 32003, 4096),
    (200, 4096, 512), (120, 40000, 128), (600, 12800, 256), (2100, 8192, 256),
]


@pytest.mark.parametrize("m,n,k", LINEAR_SHAPES)
def test_linear_accumulators_and_dequant_bit_exact(K, m, n, k):
    gen = torch.Generator().manual_seed(m * 131 + n + k)
    qa, qw = _rand_q(gen, m, k), _rand_q(gen, n, k)
    sa = O.scale_from_absmax(torch.rand(m, generator=gen).numpy() * 10 + 0.01)
    sw = O.scale_from_absmax(torch.rand(n, generator=gen).numpy() * 2 + 0.01)
    bias = (torch.randn(n, generator=gen) * 0.1).numpy()
    acc_d = torch.empty((m, n), dtype=torch.int32, device=K.dev)
    out = K.W.linear_q(qa.to(K.dev), torch.from_numpy(sa).to(K.dev), qw.to(K.dev), torch.from_numpy(sw).to(K.dev),
                       bias=torch.from_numpy(bias).to(K.dev), out_dtype=torch.float32, acc_out=acc_d)
    acc = O.int_matmul_nt(qa.numpy(), qw.numpy())
    np.testing.assert_array_equal(cpu(acc_d), acc)
    np.testing.assert_array_equal(cpu(out), O.dequantize(acc, sa, sw, bias))


@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (8, 4096, 4096), (8, 4096, 11008), (64, 512, 1024), (5, 384, 256),
                                   (300, 640, 512), (1100, 256, 256),  # prefill tiles, ragged last tile
                                   (2100, 8192, 256)])  # data-parallel waves + stream-K tail
def test_linear_residual_epilogue(K, m, n, k):
    gen = torch.Generator().manual_seed(m + n + k + 1)
    qa, qw = _rand_q(gen, m, k), _rand_q(gen, n, k)
    sa = O.scale_from_absmax(torch.rand(m, generator=gen).numpy() * 4 + 0.01)
    sw = O.scale_from_absmax(torch.rand(n, generator=gen).numpy() * 0.05 + 0.001)
    res = torch.randn(m, n, generator=gen).half()
    out = K.W.linear_q(qa.to(K.dev), torch.from_numpy(sa).to(K.dev), qw.to(K.dev), torch.from_numpy(sw).to(K.dev),
                       epilogue=K.lib.EPI_RESIDUAL, residual=res.to(K.dev))
    o16, _ = O.w8a8_linear(qa.numpy(), sa, qw.numpy(), sw)
    ref = (o16.astype(np.float32) + res.numpy().astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(cpu(out), ref)


@pytest.mark.parametrize("m,inter,k", [(1, 11008, 4096), (8, 11008, 4096), (64, 1024, 512), (5, 128, 256),
                                       (300, 1024, 512), (2100, 4096, 256)])
def test_linear_silu_mul_epilogue(K, m, inter, k):
    gen = torch.Generator().manual_seed(m + inter + k)
    qa = _rand_q(gen, m, k)
    qg, qu = _rand_q(gen, inter, k), _rand_q(gen, inter, k)
    sa = O.scale_from_absmax(torch.rand(m, generator=gen).numpy() * 4 + 0.01)
    sg = O.scale_from_absmax(torch.rand(inter, generator=gen).numpy() * 0.05 + 0.001)
    su = O.scale_from_absmax(torch.rand(inter, generator=gen).numpy() * 0.05 + 0.001)
    packed_w = K.W.pack_gate_up(qg, qu)
    packed_s = K.W.pack_gate_up(torch.from_numpy(sg), torch.from_numpy(su))
    out = K.W.linear_q(qa.to(K.dev), torch.from_numpy(sa).to(K.dev), packed_w.to(K.dev), packed_s.to(K.dev),
                       epilogue=K.lib.EPI_SILU_MUL)
    g16, _ = O.w8a8_linear(qa.numpy(), sa, qg.numpy(), sg)
    u16, _ = O.w8a8_linear(qa.numpy(), sa, qu.numpy(), su)
    np.testing.assert_array_equal(cpu(out), O.silu_mul(g16, u16))


def test_silu_mul_against_reference_fixture(K):
    """The epilogue's SiLU*up on the reference's fp16 gate/up values: within
    one fp16 ulp of torch's fp32 SiLU on <= 0.1% of elements."""
    g = golden("silu_mul.npz")
    mine = O.silu_mul(g["gate"], g["up"])  # kernel == oracle is asserted above
    d = mine.view(np.int16).astype(np.int32) - g["h"].view(np.int16).astype(np.int32)
    assert np.abs(d).max() <= 1 and (d != 0).mean() <= 1e-3


def test_linear_workspace_left_clean(K):
    """Stream-K partial tiles reduce through the workspace; repeated calls
    give identical results and leave it zero."""
    gen = torch.Generator().manual_seed(5)
    m, n, k = 8, 4096, 11008
    qa, qw = _rand_q(gen, m, k).to(K.dev), _rand_q(gen, n, k).to(K.dev)
    sa = torch.ones(m, device=K.dev)
    sw = torch.ones(n, device=K.dev)
    a1 = torch.empty((m, n), dtype=torch.int32, device=K.dev)
    a2 = torch.empty_like(a1)
    K.W.linear_q(qa, sa, qw, sw, acc_out=a1)
    K.W.linear_q(qa, sa, qw, sw, acc_out=a2)
    torch.cuda.synchronize()
    assert torch.equal(a1, a2)
    ws = K.W.linear_workspace(K.dev, m, n, k)
    assert int(ws.count_nonzero()) == 0
    K.lib.device_status()


def test_linear_argument_errors(K):
    qa = torch.zeros(8, 4096, dtype=torch.int8, device=K.dev)
    sa = torch.ones(8, device=K.dev)
    with pytest.raises(ValueError):
        K.W.linear_q(qa, sa, torch.zeros(16, 4000, dtype=torch.int8, device=K.dev), torch.ones(16, device=K.dev))
    big_k = 133152  # K * 127^2 >= 2^31
    with pytest.raises(OverflowError):
        K.W.linear_q(torch.zeros(1, big_k, dtype=torch.int8, device=K.dev), sa[:1],
                     torch.zeros(16, big_k, dtype=torch.int8, device=K.dev), torch.ones(16, device=K.dev))


# ------------------------------------------------------------- RoPE / KV
@pytest.mark.parametrize("pad", [0, 4])  # 0: 16-byte rows (vector kernel); 4: row stride not a multiple of 8
def test_rope_store_bit_exact(K, pad):
    g = golden("rope.npz")
    t, h, d = g["q"].shape
    hkv = g["k"].shape[1]
    # tables holding the reference's own cos/sin rows at the fixture positions
    # (torch's CPU cos/sin may round differently on another host CPU)
    cos = np.zeros((4096, d), np.float16)
    sin = np.zeros((4096, d), np.float16)
    cos[g["positions"]] = g["cos"]
    sin[g["positions"]] = g["sin"]
    qkv = np.concatenate([g["q"].reshape(t, -1), g["k"].reshape(t, -1), g["k"].reshape(t, -1) * 0.5], 1)
    qkv_dev = torch.zeros(t, qkv.shape[1] + pad, dtype=torch.float16, device=K.dev)
    qkv_dev[:, :qkv.shape[1]] = torch.from_numpy(qkv).to(K.dev)
    nb, bs = 4, 4
    kc = torch.zeros(nb, bs, hkv, d, dtype=torch.float16, device=K.dev)
    vc = torch.zeros_like(kc)
    slots = torch.tensor([3, 0, -1, 5, 6, 7, 8, 15], dtype=torch.int32, device=K.dev)
    q = K.PA.rope_store_kvcache(qkv_dev[:, :qkv.shape[1]], h, hkv, d, torch.from_numpy(cos).to(K.dev),
                                torch.from_numpy(sin).to(K.dev), torch.from_numpy(g["positions"]).to(K.dev),
                                slots, kc, vc)
    np.testing.assert_array_equal(cpu(q), g["q_rot"])
    kcn, vcn = cpu(kc), cpu(vc)
    for i, s in enumerate(cpu(slots).tolist()):
        if s < 0:
            continue
        np.testing.assert_array_equal(kcn[s // bs, s % bs], g["k_rot"][i])
        np.testing.assert_array_equal(vcn[s // bs, s % bs], qkv[i, (h + hkv) * d:].reshape(hkv, d))
    assert float(kcn[0, 2].astype(np.float32).sum()) == 0.0  # slot 2 never written (padding row)


def test_rope_store_vector_and_scalar_kernels_agree(K):
    """Prefill-sized batch (300 tokens, GQA 8/2, D = 128): the 16-byte vector
    kernel (contiguous rows) and the scalar kernel (row stride not a multiple
    of 8) write identical q, k and v bits."""
    gen = torch.Generator().manual_seed(11)
    t, h, hkv, d, nb, bs = 300, 8, 2, 128, 24, 16
    cols = (h + 2 * hkv) * d
    qkv = (torch.randn(t, cols + 4, generator=gen) * 3).half().to(K.dev)
    cos = torch.randn(512, d, generator=gen).half().to(K.dev)
    sin = torch.randn(512, d, generator=gen).half().to(K.dev)
    pos = torch.randint(0, 512, (t,), generator=gen).to(K.dev)
    slots = torch.randperm(nb * bs, generator=gen)[:t].to(torch.int32).to(K.dev)
    outs = []
    for view in (qkv[:, :cols].contiguous(), qkv[:, :cols]):
        kc = torch.zeros(nb, bs, hkv, d, dtype=torch.float16, device=K.dev)
        vc = torch.zeros_like(kc)
        outs.append((K.PA.rope_store_kvcache(view, h, hkv, d, cos, sin, pos, slots, kc, vc), kc, vc))
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_store_kvcache_reference_cases(K):
    # tests/test_store_kvcache.py patterns: contiguous, scattered, padding, single token
    kc = torch.zeros(4, 4, 2, 8, dtype=torch.float16, device=K.dev)
    vc = torch.zeros_like(kc)
    key = torch.arange(4 * 2 * 8, dtype=torch.float16, device=K.dev).reshape(4, 2, 8)
    K.PA.store_kvcache(key, -key, kc, vc, torch.tensor([-1, 5, -1, 12], dtype=torch.int32, device=K.dev))
    assert torch.equal(kc[1, 1], key[1]) and torch.equal(kc[3, 0], key[3]) and torch.equal(vc[3, 0], -key[3])
    assert float(kc.abs().sum()) == float(key[1].abs().sum() + key[3].abs().sum())
    K.PA.store_kvcache(key[:1], key[:1], kc, vc, torch.tensor([7], dtype=torch.int32, device=K.dev))
    assert torch.equal(kc[1, 3], key[0])


# --------------------------------------------------------------- attention
def test_decode_attention_reference_fixture(K):
    g = golden("decode_attention.npz")
    dev = K.dev
    out = K.PA.paged_decode_attention(
        torch.from_numpy(g["q"]).to(dev), torch.from_numpy(g["k_cache"]).to(dev),
        torch.from_numpy(g["v_cache"]).to(dev), torch.from_numpy(g["block_tables"]).to(dev),
        torch.from_numpy(g["context_lens"]).to(dev), float(g["scale"]), int(g["groups"]))
    # fp16 output of an fp32-accumulated softmax: |err| <= 2e-3 (one fp16 ulp at 1.0 is 9.8e-4)
    np.testing.assert_allclose(cpu(out).astype(np.float32), g["out"], atol=2e-3, rtol=2e-3)


@pytest.mark.parametrize("b,h,hkv,bs,ctx", [
    (8, 32, 32, 256, [1024, 1087, 1000, 1, 0, 257, 512, 768]),  # 7B decode, incl. a padded row (ctx 0)
    (3, 8, 2, 16, [5, 70, 33]),
    (2, 4, 4, 64, [300, 64]),
    (3, 64, 8, 32, [700, 33, 0]),    # 4 heads per consumer warp (16 dims per lane)
    (2, 48, 16, 16, [300, 64]),      # 12 consumer warps, 8-token stages
    (2, 6, 2, 16, [90, 200]),        # H not a multiple of 4: the per-head kernel
    (2, 8, 8, 256, [1, 2]),
])
def test_decode_attention_vs_oracle(K, b, h, hkv, bs, ctx):
    d = 128
    gen = torch.Generator().manual_seed(b * h + bs)
    blocks = [max(1, (n + bs - 1) // bs) for n in ctx]
    mb = max(blocks) + 1
    nb = b * mb + 3
    from nanopointllm_b200 import synthetic as S
    bt = S.permuted_block_tables(b, mb, nb, seed=bs)
    kc = (torch.randn(nb, bs, hkv, d, generator=gen)).half()
    vc = (torch.randn(nb, bs, hkv, d, generator=gen)).half()
    q = torch.randn(b, h, d, generator=gen).half()
    ctx_t = torch.tensor(ctx, dtype=torch.int32)
    out = K.PA.paged_decode_attention(q.to(K.dev), kc.to(K.dev), vc.to(K.dev), bt.to(K.dev), ctx_t.to(K.dev),
                                      d ** -0.5, h // hkv)
    ref = O.paged_decode_attention(q.numpy(), kc.numpy(), vc.numpy(), bt.numpy(), ctx, d ** -0.5, h // hkv)
    got = cpu(out).astype(np.float64)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, atol=2e-3, rtol=2e-3)
    # a second call reuses the workspace
    out2 = K.PA.paged_decode_attention(q.to(K.dev), kc.to(K.dev), vc.to(K.dev), bt.to(K.dev), ctx_t.to(K.dev),
                                       d ** -0.5, h // hkv)
    assert torch.equal(out, out2)
    K.lib.device_status()


def test_decode_attention_shared_workspace(K):
    """Calls of different shapes share one workspace and each stays within
    tolerance of the oracle, with the fused per-token quantisation; repeated
    shapes give identical outputs; every call leaves the workspace's counters
    and flags zero."""
    from nanopointllm_b200 import synthetic as S
    prev = {}
    for b, h, mb, ctx in ((8, 32, 6, 1087), (2, 4, 2, 20), (4, 8, 3, 500), (1, 2, 40, 9000), (8, 32, 6, 1087)):
        bs = 256
        g2 = torch.Generator().manual_seed(b * 1000 + ctx)
        kc = torch.randn(b * mb, bs, h, 128, generator=g2).half()
        vc = torch.randn(b * mb, bs, h, 128, generator=g2).half()
        q = torch.randn(b, h, 128, generator=g2).half()
        bt = S.permuted_block_tables(b, mb, b * mb, seed=b)
        ctx_l = [ctx] * b
        q8 = torch.empty((b, h * 128), dtype=torch.int8, device=K.dev)
        qs = torch.empty((b,), dtype=torch.float32, device=K.dev)
        out = K.PA.paged_decode_attention(q.to(K.dev), kc.to(K.dev), vc.to(K.dev), bt.to(K.dev),
                                          torch.tensor(ctx_l, dtype=torch.int32, device=K.dev), 128 ** -0.5, 1,
                                          quant_out=(q8, qs))
        ref = O.paged_decode_attention(q.numpy(), kc.numpy(), vc.numpy(), bt.numpy(), ctx_l, 128 ** -0.5, 1)
        np.testing.assert_allclose(cpu(out).astype(np.float64), ref, atol=2e-3, rtol=2e-3)
        key = (b, h, mb, ctx)
        if key in prev:
            assert torch.equal(prev[key], out)
        prev[key] = out
        # the counters and flags at the front of the workspace (work counters,
        # 1024 sequence counters, 2^18 chunk flags) are zero after every call
        torch.cuda.synchronize()
        ws = K.PA.decode_attention_workspace(K.dev, b, h, 128, mb, bs)
        assert int(ws[:256 + 4096 + (4 << 18)].count_nonzero()) == 0
    K.lib.device_status()


def test_decode_attention_ragged_batch_more_units_than_sms(K):
    """A ragged batch of 40 sequences has more 64-token units than the GPU
    has SMs, so the units are handed out by the work counter: the output stays
    within tolerance of the oracle, the fused int8 rows equal npl_quant_rows
    on it, each sequence's row equals the row it gets alone in a batch of one
    (batch invariance, bit for bit), and the workspace counters are zero
    afterwards."""
    from nanopointllm_b200 import synthetic as S
    b, h, hkv, d, bs = 40, 32, 8, 128, 64
    gen = torch.Generator().manual_seed(23)
    ctx = torch.randint(2, 1500, (b,), generator=gen).tolist()
    ctx[:6] = [0, 1, 64, 65, 1500, 128]
    assert sum(max(1, -(-n // 64)) for n in ctx) > 200
    mb = -(-max(ctx) // bs) + 1
    nb = b * mb
    kc = torch.randn(nb, bs, hkv, d, generator=gen).half()
    vc = torch.randn(nb, bs, hkv, d, generator=gen).half()
    q = torch.randn(b, h, d, generator=gen).half()
    bt = S.permuted_block_tables(b, mb, nb, seed=5)
    dev = K.dev
    kcd, vcd, btd = kc.to(dev), vc.to(dev), bt.to(dev)
    q8 = torch.empty((b, h * d), dtype=torch.int8, device=dev)
    qs = torch.empty((b,), dtype=torch.float32, device=dev)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
    out = K.PA.paged_decode_attention(q.to(dev), kcd, vcd, btd, ctx_d, d ** -0.5, h // hkv, quant_out=(q8, qs))
    ref = O.paged_decode_attention(q.numpy(), kc.numpy(), vc.numpy(), bt.numpy(), ctx, d ** -0.5, h // hkv)
    np.testing.assert_allclose(cpu(out).astype(np.float64), ref, atol=2e-3, rtol=2e-3)
    ref_q, ref_s = K.W.dynamic_per_token_quant(out.reshape(b, -1))
    torch.cuda.synchronize()
    assert torch.equal(q8, ref_q) and torch.equal(qs, ref_s.reshape(-1))
    assert float(out[0].abs().sum()) == 0.0
    ws = K.PA.decode_attention_workspace(dev, b, h, d, mb, bs)
    assert int(ws[:256 + 4096 + (4 << 18)].count_nonzero()) == 0
    for i in (0, 1, 3, 4, 17, 39):
        alone = K.PA.paged_decode_attention(q[i:i + 1].to(dev), kcd, vcd, btd[i:i + 1].contiguous(),
                                            ctx_d[i:i + 1].contiguous(), d ** -0.5, h // hkv)
        assert torch.equal(alone[0], out[i]), f"sequence {i}"
    out2 = K.PA.paged_decode_attention(q.to(dev), kcd, vcd, btd, ctx_d, d ** -0.5, h // hkv)
    assert torch.equal(out, out2)
    K.lib.device_status()


def test_decode_attention_fused_quant_equals_quant_rows(K):
    """The per-token int8 quantisation fused into the attention kernel equals
    npl_quant_rows on the attention's own fp16 output, bit for bit (including
    a padded row with context 0)."""
    from nanopointllm_b200 import synthetic as S
    gen = torch.Generator().manual_seed(17)
    b, h, d, bs, mb = 8, 32, 128, 256, 5
    nb = b * mb
    kc = torch.randn(nb, bs, h, d, generator=gen).half().to(K.dev)
    vc = torch.randn(nb, bs, h, d, generator=gen).half().to(K.dev)
    q = torch.randn(b, h, d, generator=gen).half().to(K.dev)
    bt = S.permuted_block_tables(b, mb, nb, seed=2).to(K.dev)
    ctx = torch.tensor([1024, 1087, 0, 1, 300, 256, 257, 1280], dtype=torch.int32, device=K.dev)
    q8 = torch.empty((b, h * d), dtype=torch.int8, device=K.dev)
    qs = torch.empty((b,), dtype=torch.float32, device=K.dev)
    for _ in range(2):
        out = K.PA.paged_decode_attention(q, kc, vc, bt, ctx, d ** -0.5, 1, quant_out=(q8, qs))
        ref_q, ref_s = K.W.dynamic_per_token_quant(out.reshape(b, -1))
        torch.cuda.synchronize()
        assert torch.equal(q8, ref_q)
        assert torch.equal(qs, ref_s.reshape(-1))
    assert float(out[2].abs().sum()) == 0.0
    K.lib.device_status()


@pytest.mark.parametrize("h,hkv,bs,ctx", [(4, 4, 16, [38, 65, 21]), (32, 32, 256, [1025, 1, 0, 700])])
def test_decode_attention_right_after_rope_store(K, h, hkv, bs, ctx):
    """The runner's order: RoPE + KV store writes q and the new token's K/V,
    then the attention (launched early behind it) reads them, with the fused
    per-token quantisation; against the oracle on the same q and pool."""
    from nanopointllm_b200 import synthetic as S
    d, b = 128, len(ctx)
    gen = torch.Generator().manual_seed(h + bs)
    mb = max(1, max(-(-n // bs) for n in ctx)) + 1
    nb = b * mb + 2
    bt = S.permuted_block_tables(b, mb, nb, seed=bs).to(K.dev)
    kc = torch.randn(nb, bs, hkv, d, generator=gen).half().to(K.dev)
    vc = torch.randn(nb, bs, hkv, d, generator=gen).half().to(K.dev)
    qkv = torch.randn(b, (h + 2 * hkv) * d, generator=gen).half().to(K.dev)
    from nanopointllm_b200.rope import rope_tables
    cos, sin = rope_tables(d, 4096, 10000.0, K.dev)
    ctx_t = torch.tensor(ctx, dtype=torch.int32, device=K.dev)
    pos = (ctx_t.long() - 1).clamp_min(0)
    slots = torch.tensor([int(bt[i, max(n - 1, 0) // bs]) * bs + max(n - 1, 0) % bs if n > 0 else -1
                          for i, n in enumerate(ctx)], dtype=torch.int32, device=K.dev)
    for _ in range(2):
        q = K.PA.rope_store_kvcache(qkv, h, hkv, d, cos, sin, pos, slots, kc, vc)
        q8 = torch.empty((b, h * d), dtype=torch.int8, device=K.dev)
        qs = torch.empty((b,), dtype=torch.float32, device=K.dev)
        out = K.PA.paged_decode_attention(q, kc, vc, bt, ctx_t, d ** -0.5, h // hkv, quant_out=(q8, qs))
        torch.cuda.synchronize()
        ref = O.paged_decode_attention(cpu(q), cpu(kc), cpu(vc), cpu(bt), ctx, d ** -0.5, h // hkv)
        np.testing.assert_allclose(cpu(out).astype(np.float64), ref, atol=2e-3, rtol=2e-3)
        ref_q, ref_s = K.W.dynamic_per_token_quant(out.reshape(b, -1))
        assert torch.equal(q8, ref_q)
        assert torch.equal(qs, ref_s.reshape(-1))
    K.lib.device_status()
