"""npl_w8a8_linear_ex on the GPU: the decode linear with RMSNorm + activation
quantisation fused before it and RoPE + KV store / SiLU*up + absmax /
residual after it. Every output must equal the oracle's unfused sequence bit
for bit (the same numerics as the separate kernels)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import w8a8 as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K(cuda_device):
    from nanopointllm_b200 import _lib, paged_attention, w8a8
    return type("K", (), dict(lib=_lib, W=w8a8, PA=paged_attention, dev=cuda_device))


def cpu(t):
    return t.detach().cpu().numpy()


def _qweight(gen, n, k, std=0.02):
    w = (torch.randn(n, k, generator=gen) * std).half()
    return O.per_output_weight_quant(w.numpy())


@pytest.mark.parametrize("m,n,k", [(1, 1000, 4096), (8, 12288, 4096), (33, 384, 512), (64, 640, 1024)])
def test_rmsnorm_fused_linear_bit_exact(K, m, n, k):
    gen = torch.Generator().manual_seed(m * 3 + n + k)
    x = torch.randn(m, k, generator=gen).half()
    w = (1 + 0.1 * torch.randn(k, generator=gen)).half()
    qw, sw = _qweight(gen, n, k)
    acc = torch.empty((m, n), dtype=torch.int32, device=K.dev)
    out = K.W.linear_ex(torch.from_numpy(qw).to(K.dev), torch.from_numpy(sw).to(K.dev), x_mode=K.lib.X_F16_RMSNORM,
                        m=m, x_f16=x.to(K.dev), norm_weight=w.to(K.dev), eps=1e-6, acc_out=acc)
    q8, s8, _, _ = O.rmsnorm_quant(x.numpy(), w.numpy(), 1e-6)
    ref, ref_acc = O.w8a8_linear(q8, s8, qw, sw)
    np.testing.assert_array_equal(cpu(acc), ref_acc)
    np.testing.assert_array_equal(cpu(out), ref)


@pytest.mark.parametrize("m,h,hkv", [(8, 4, 2), (3, 4, 4), (16, 8, 8)])
def test_qkv_rope_kv_epilogue_bit_exact(K, m, h, hkv):
    d, k, nb, bs = 128, 512, 6, 16
    gen = torch.Generator().manual_seed(m + h + hkv)
    n = (h + 2 * hkv) * d
    x = torch.randn(m, k, generator=gen).half()
    w = (1 + 0.1 * torch.randn(k, generator=gen)).half()
    qw, sw = _qweight(gen, n, k)
    cos, sin = O.rope_tables(np.arange(256), d)
    pos = torch.randint(0, 256, (m,), generator=gen)
    slots = torch.randperm(nb * bs, generator=gen)[:m].to(torch.int32)
    slots[m // 2] = -1  # a padded row: nothing stored
    kc0 = torch.randn(nb, bs, hkv, d, generator=gen).half()
    vc0 = torch.randn(nb, bs, hkv, d, generator=gen).half()
    kc, vc = kc0.clone().to(K.dev), vc0.clone().to(K.dev)
    q_out = torch.empty((m, h, d), dtype=torch.float16, device=K.dev)
    rope = dict(cos=torch.from_numpy(cos).to(K.dev), sin=torch.from_numpy(sin).to(K.dev), positions=pos.to(K.dev),
                slots=slots.to(K.dev), q_out=q_out, k_cache=kc, v_cache=vc, heads=h, kv_heads=hkv, head_dim=d)
    K.W.linear_ex(torch.from_numpy(qw).to(K.dev), torch.from_numpy(sw).to(K.dev), x_mode=K.lib.X_F16_RMSNORM, m=m,
                  x_f16=x.to(K.dev), norm_weight=w.to(K.dev), eps=1e-6, epilogue=K.lib.EPI_ROPE_KV, rope=rope)
    q8, s8, _, _ = O.rmsnorm_quant(x.numpy(), w.numpy(), 1e-6)
    qkv, _ = O.w8a8_linear(q8, s8, qw, sw)
    qh = qkv[:, : h * d].reshape(m, h, d)
    kh = qkv[:, h * d:(h + hkv) * d].reshape(m, hkv, d)
    vh = qkv[:, (h + hkv) * d:].reshape(m, hkv, d)
    c, sn = cos[pos.numpy()], sin[pos.numpy()]
    ref_q = O.apply_rope(qh, c, sn)
    ref_k = O.apply_rope(kh, c, sn)
    kref, vref = kc0.numpy().copy(), vc0.numpy().copy()
    O.store_kvcache(ref_k, vh, kref, vref, slots.numpy())
    np.testing.assert_array_equal(cpu(q_out), ref_q)
    np.testing.assert_array_equal(cpu(kc), kref)
    np.testing.assert_array_equal(cpu(vc), vref)


def _mlp_oracle(x, nw, qg, sg, qu, su, qd, sd):
    q8, s8, _, _ = O.rmsnorm_quant(x, nw, 1e-6)
    g16, _ = O.w8a8_linear(q8, s8, qg, sg)
    u16, _ = O.w8a8_linear(q8, s8, qu, su)
    h = O.silu_mul(g16, u16)
    hq, hs = O.dynamic_per_token_quant(h)
    d16, _ = O.w8a8_linear(hq, hs, qd, sd)
    return h, (d16.astype(np.float32) + x.astype(np.float32)).astype(np.float16)


@pytest.mark.parametrize("m", [1, 8, 32, 64])
def test_mlp_block_config2_runner_sequence(K, m):
    """BASELINE config 2 (Llama-7B decode MLP block, M in {1, 8, 32, 64}) the
    way the decode runner runs it: fused RMSNorm + per-token quant kernel,
    packed gate/up with SiLU(gate)*up in its epilogue, per-token requant,
    down with the residual add in its epilogue; bit-exact against the
    oracle."""
    from nanopointllm_b200 import runner as R
    from nanopointllm_b200 import synthetic as S
    x, _, nw, gate, up, down = S.mlp_block_inputs(m, seed=1)
    qg, sg = O.per_output_weight_quant(gate.numpy())
    qu, su = O.per_output_weight_quant(up.numpy())
    qd, sd = O.per_output_weight_quant(down.numpy())
    dev = K.dev
    packed_w = K.W.pack_gate_up(torch.from_numpy(qg), torch.from_numpy(qu)).to(dev)
    packed_s = K.W.pack_gate_up(torch.from_numpy(sg), torch.from_numpy(su)).to(dev)
    xd = x.to(dev)
    xq, xs, _ = R.rmsnorm_quant(xd, nw.to(dev), 1e-6)
    act = K.W.linear_q(xq, xs, packed_w, packed_s, epilogue=K.lib.EPI_SILU_MUL)
    aq, asc = K.W.dynamic_per_token_quant(act)
    out = K.W.linear_q(aq, asc.reshape(-1), torch.from_numpy(qd).to(dev), torch.from_numpy(sd).to(dev),
                       epilogue=K.lib.EPI_RESIDUAL, residual=xd)
    h, ref = _mlp_oracle(x.numpy(), nw.numpy(), qg, sg, qu, su, qd, sd)
    np.testing.assert_array_equal(cpu(act), h)
    np.testing.assert_array_equal(cpu(out), ref)


@pytest.mark.parametrize("m", [1, 8, 32])
def test_mlp_block_config2_fused_activations(K, m):
    """The same block through npl_w8a8_linear_ex's fp16-activation modes:
    RMSNorm + per-token int8 quantisation inside packed gate/up, SiLU(gate)*up
    + per-token absmax in its epilogue, re-quantisation inside down, residual
    add in its epilogue; bit-exact against the oracle's unfused sequence."""
    from nanopointllm_b200 import synthetic as S
    x, _, nw, gate, up, down = S.mlp_block_inputs(m, seed=1)
    qg, sg = O.per_output_weight_quant(gate.numpy())
    qu, su = O.per_output_weight_quant(up.numpy())
    qd, sd = O.per_output_weight_quant(down.numpy())
    dev = K.dev
    packed_w = K.W.pack_gate_up(torch.from_numpy(qg), torch.from_numpy(qu)).to(dev)
    packed_s = K.W.pack_gate_up(torch.from_numpy(sg), torch.from_numpy(su)).to(dev)
    amax = torch.zeros(64, dtype=torch.int32, device=dev)
    xd = x.to(dev)
    act = K.W.linear_ex(packed_w, packed_s, x_mode=K.lib.X_F16_RMSNORM, m=m, x_f16=xd, norm_weight=nw.to(dev),
                        eps=1e-6, epilogue=K.lib.EPI_SILU_MUL, absmax_out=amax)
    torch.cuda.synchronize()
    q8, s8, _, _ = O.rmsnorm_quant(x.numpy(), nw.numpy(), 1e-6)
    g16, _ = O.w8a8_linear(q8, s8, qg, sg)
    u16, _ = O.w8a8_linear(q8, s8, qu, su)
    h = O.silu_mul(g16, u16)
    np.testing.assert_array_equal(cpu(act), h)
    ref_amax = np.abs(h.astype(np.float32)).max(axis=1).astype(np.float32).view(np.int32)
    np.testing.assert_array_equal(cpu(amax)[:m], ref_amax)
    out = K.W.linear_ex(torch.from_numpy(qd).to(dev), torch.from_numpy(sd).to(dev), x_mode=K.lib.X_F16_ABSMAX, m=m,
                        x_f16=act, x_absmax=amax, epilogue=K.lib.EPI_RESIDUAL, residual=xd)
    torch.cuda.synchronize()
    hq, hs = O.dynamic_per_token_quant(h)
    d16, _ = O.w8a8_linear(hq, hs, qd, sd)
    ref = (d16.astype(np.float32) + x.numpy().astype(np.float32)).astype(np.float16)
    np.testing.assert_array_equal(cpu(out), ref)
    assert int(amax.count_nonzero()) == 0  # consumed: zeroed for the next producer
    K.lib.device_status()


def test_fp16_activations_limited_to_decode_batches(K):
    qw = torch.zeros(128, 256, dtype=torch.int8, device=K.dev)
    sw = torch.ones(128, device=K.dev)
    x = torch.zeros(65, 256, dtype=torch.float16, device=K.dev)
    with pytest.raises(K.lib.NplError):
        K.W.linear_ex(qw, sw, x_mode=K.lib.X_F16_RMSNORM, m=65, x_f16=x, norm_weight=torch.ones(256).half().to(K.dev))


@pytest.mark.parametrize("m", [1, 8, 33, 64])
def test_gate_up_quantises_its_output_in_the_same_launch(K, m):
    """Packed gate/up with q_out / q_scale: after all of its CTAs have stored
    SiLU(gate)*up, the launch quantises the rows per token itself. The int8
    rows and scales equal npl_quant_rows on the fp16 output (and the oracle),
    on two calls in a row (the grid-wide counts and the absmax words are left
    zero for the next call)."""
    from nanopointllm_b200 import synthetic as S
    x, _, nw, gate, up, _ = S.mlp_block_inputs(m, seed=2)
    qg, sg = O.per_output_weight_quant(gate.numpy())
    qu, su = O.per_output_weight_quant(up.numpy())
    dev = K.dev
    packed_w = K.W.pack_gate_up(torch.from_numpy(qg), torch.from_numpy(qu)).to(dev)
    packed_s = K.W.pack_gate_up(torch.from_numpy(sg), torch.from_numpy(su)).to(dev)
    q8, s8, _, _ = O.rmsnorm_quant(x.numpy(), nw.numpy(), 1e-6)
    g16, _ = O.w8a8_linear(q8, s8, qg, sg)
    u16, _ = O.w8a8_linear(q8, s8, qu, su)
    h = O.silu_mul(g16, u16)
    hq, hs = O.dynamic_per_token_quant(h)
    amax = torch.zeros(64, dtype=torch.int32, device=dev)
    inter = gate.shape[0]
    for _ in range(2):
        aq = torch.full((m, inter), 99, dtype=torch.int8, device=dev)
        asc = torch.zeros(m, dtype=torch.float32, device=dev)
        act = K.W.linear_ex(packed_w, packed_s, x_mode=K.lib.X_INT8, m=m, qa=torch.from_numpy(q8).to(dev),
                            sa=torch.from_numpy(s8).to(dev), epilogue=K.lib.EPI_SILU_MUL, absmax_out=amax,
                            q_out=aq, q_scale=asc)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(cpu(act), h)
        np.testing.assert_array_equal(cpu(aq), hq)
        np.testing.assert_array_equal(cpu(asc), hs.reshape(-1))
        sq, ss = K.W.dynamic_per_token_quant(act)
        assert torch.equal(sq, aq) and torch.equal(ss.reshape(-1), asc)
        assert int(amax.count_nonzero()) == 0
    K.lib.device_status()
