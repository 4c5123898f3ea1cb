"""The tensor-parallel peer-memory exchanges (npl_tp_absmax_quant,
npl_tp_allreduce_dequant) on ONE GPU, with the other rank emulated: its
pushed data and raised flags are written into this rank's exchange buffer
before the call, and a second local buffer stands in for its mapped buffer
(which receives this rank's push). Results must equal the NCCL path's kernels
(npl_row_absmax / npl_quant_rows_absmax / npl_dequant) bit for bit, over two
calls (both slot parities). A flag that nothing raises must end the wait
with device code 6 after ~1 s, not hang. Nothing here waits on another
kernel: a single launch at a time, on a single GPU."""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD, RANK, PEER = 2, 0, 1
SUM_CTAS, MAX_ROWS, MAX_RANKS = 64, 64, 8


def layout(world: int, max_elems: int) -> dict[str, int]:
    """Byte offsets of the exchange buffer (tp_exchange.cu x_layout)."""
    al = lambda x: (x + 255) & ~255  # noqa: E731
    lay = {"flags_sum": 0}
    lay["flags_max"] = lay["flags_sum"] + al(4 * MAX_RANKS * SUM_CTAS)
    lay["seen_sum"] = lay["flags_max"] + al(4 * MAX_RANKS * MAX_ROWS)
    lay["seen_max"] = lay["seen_sum"] + al(4 * SUM_CTAS)
    lay["data_sum"] = lay["seen_max"] + al(4 * MAX_ROWS)
    lay["data_max"] = lay["data_sum"] + al(4 * 2 * world * max_elems)
    lay["total"] = lay["data_max"] + al(4 * 2 * world * MAX_ROWS)
    return lay


def i32(buf: torch.Tensor, off: int, n: int) -> torch.Tensor:
    return buf[off:off + 4 * n].view(torch.int32)


def make_peers(own: torch.Tensor, peer: torch.Tensor, max_elems: int):
    from nanopointllm_b200 import _lib as L
    ptrs = [own.data_ptr(), peer.data_ptr()] + [0] * (L.TP_MAX_RANKS - 2)
    return L.NplTpPeers(WORLD, RANK, (ctypes.c_void_p * L.TP_MAX_RANKS)(*ptrs), max_elems)


@pytest.fixture
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    d = torch.device("cuda:0")
    torch.cuda.set_device(d)
    return d


def test_allreduce_dequant_matches_nccl_path_kernels(dev):
    from nanopointllm_b200 import _lib as L, w8a8 as W
    m, n = 8, 4096
    max_elems = MAX_ROWS * n
    lay = layout(WORLD, max_elems)
    nbytes = int(L.lib.npl_tp_exchange_bytes(WORLD, max_elems))
    assert nbytes == lay["total"]
    own = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    fake_peer = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    peers = make_peers(own, fake_peer, max_elems)
    g = torch.Generator(device=dev).manual_seed(0)
    sa = (torch.rand(m, generator=g, device=dev) * 1e-2 + 1e-4).float()
    sw = (torch.rand(n, generator=g, device=dev) * 1e-3 + 1e-5).float()
    residual = torch.randn(m, n, generator=g, device=dev).half()
    stream = L.stream_ptr(dev)
    for call in (1, 2):  # sequence numbers 1 and 2: both parities of the data slots
        par = call & 1
        acc0 = torch.randint(-2 ** 24, 2 ** 24, (m, n), generator=g, device=dev, dtype=torch.int32)
        acc1 = torch.randint(-2 ** 24, 2 ** 24, (m, n), generator=g, device=dev, dtype=torch.int32)
        # the emulated peer's push into our buffer, and its flags
        i32(own, lay["data_sum"] + 4 * (par * WORLD + PEER) * max_elems, m * n).copy_(acc1.reshape(-1))
        i32(own, lay["flags_sum"] + 4 * PEER * SUM_CTAS, SUM_CTAS).fill_(call)
        out = torch.empty(m, n, dtype=torch.float16, device=dev)
        L.check(L.lib.npl_tp_allreduce_dequant(ctypes.byref(peers), acc0.data_ptr(), m, n, sa.data_ptr(),
                                               sw.data_ptr(), None, residual.data_ptr(), n, out.data_ptr(), n,
                                               stream))
        ref = W.dequant(acc0 + acc1, sa, sw, residual=residual)
        torch.cuda.synchronize()
        L.device_status()
        assert torch.equal(out, ref)
        # our partials and flags landed in the emulated peer's buffer
        got = i32(fake_peer, lay["data_sum"] + 4 * (par * WORLD + RANK) * max_elems, m * n)
        assert torch.equal(got, acc0.reshape(-1))
        assert torch.all(i32(fake_peer, lay["flags_sum"] + 4 * RANK * SUM_CTAS, SUM_CTAS) == call)
        assert torch.all(i32(own, lay["seen_sum"], SUM_CTAS) == call)


def test_absmax_quant_matches_nccl_path_kernels(dev):
    from nanopointllm_b200 import _lib as L, w8a8 as W
    m, k = 8, 2048
    max_elems = MAX_ROWS * 4096
    lay = layout(WORLD, max_elems)
    nbytes = int(L.lib.npl_tp_exchange_bytes(WORLD, max_elems))
    own = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    fake_peer = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    peers = make_peers(own, fake_peer, max_elems)
    g = torch.Generator(device=dev).manual_seed(1)
    stream = L.stream_ptr(dev)
    for call in (1, 2):
        par = call & 1
        x = torch.randn(m, k, generator=g, device=dev).half()
        x[0] *= 30  # rows whose max is local, rows whose max is the peer's
        peer_amax = (torch.rand(m, generator=g, device=dev) * 8).float()
        i32(own, lay["data_max"] + 4 * (par * WORLD + PEER) * MAX_ROWS, m).copy_(peer_amax.view(torch.int32))
        i32(own, lay["flags_max"] + 4 * PEER * MAX_ROWS, m).fill_(call)
        q = torch.empty(m, k, dtype=torch.int8, device=dev)
        s = torch.empty(m, dtype=torch.float32, device=dev)
        L.check(L.lib.npl_tp_absmax_quant(ctypes.byref(peers), x.data_ptr(), m, k, k, q.data_ptr(), k,
                                          s.data_ptr(), stream))
        local = W.row_absmax(x).view(torch.float32)
        whole = torch.maximum(local, peer_amax)
        q_ref, s_ref = W.quant_rows_absmax(x, whole.view(torch.int32))
        torch.cuda.synchronize()
        L.device_status()
        assert torch.equal(q, q_ref)
        assert torch.equal(s, s_ref.reshape(-1))
        sent = i32(fake_peer, lay["data_max"] + 4 * (par * WORLD + RANK) * MAX_ROWS, m).view(torch.float32)
        assert torch.equal(sent, local)


def test_exchange_wait_is_bounded(dev):
    """No peer raises the flags: every CTA gives up after ~1 s, records device
    code 6 and leaves the output unwritten; the context stays usable."""
    from nanopointllm_b200 import _lib as L
    m, n = 8, 256
    max_elems = MAX_ROWS * n
    nbytes = int(L.lib.npl_tp_exchange_bytes(WORLD, max_elems))
    own = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    fake_peer = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    peers = make_peers(own, fake_peer, max_elems)
    acc = torch.ones(m, n, dtype=torch.int32, device=dev)
    sa = torch.ones(m, device=dev)
    sw = torch.ones(n, device=dev)
    out = torch.full((m, n), 7.0, dtype=torch.float16, device=dev)
    L.device_status()  # clear
    L.check(L.lib.npl_tp_allreduce_dequant(ctypes.byref(peers), acc.data_ptr(), m, n, sa.data_ptr(), sw.data_ptr(),
                                           None, None, 0, out.data_ptr(), n, L.stream_ptr(dev)))
    torch.cuda.synchronize()
    code = ctypes.c_int(0)
    L.lib.npl_device_status(ctypes.byref(code), 1)
    assert code.value == 6
    assert torch.all(out == 7.0)
    x = torch.randn(4, 4, device=dev)
    assert torch.isfinite((x @ x).sum()).item()  # the context still works


def test_exchange_argument_checks(dev):
    from nanopointllm_b200 import _lib as L
    max_elems = MAX_ROWS * 256
    own = torch.zeros(int(L.lib.npl_tp_exchange_bytes(WORLD, max_elems)), dtype=torch.uint8, device=dev)
    peers = make_peers(own, own, max_elems)
    acc = torch.zeros(65, 256, dtype=torch.int32, device=dev)
    out = torch.empty(65, 256, dtype=torch.float16, device=dev)
    s = torch.ones(256, device=dev)
    with pytest.raises(ValueError):  # M * N beyond the buffer
        L.check(L.lib.npl_tp_allreduce_dequant(ctypes.byref(peers), acc.data_ptr(), 65, 256, s.data_ptr(),
                                               s.data_ptr(), None, None, 0, out.data_ptr(), 256, L.stream_ptr(dev)))
    bad = L.NplTpPeers(9, 0, (ctypes.c_void_p * L.TP_MAX_RANKS)(), max_elems)
    with pytest.raises(ValueError):  # world beyond NPL_TP_MAX_RANKS
        L.check(L.lib.npl_tp_allreduce_dequant(ctypes.byref(bad), acc.data_ptr(), 1, 256, s.data_ptr(),
                                               s.data_ptr(), None, None, 0, out.data_ptr(), 256, L.stream_ptr(dev)))
