// Tensor-parallel exchanges over NVLink peer memory, fused with the work on
// either side of them.
//
// A row-parallel linear (O, down) of the tensor-parallel runner needs two
// exchanges: the per-token absmax of the whole input row (a MAX over the
// ranks, because the int8 scale is that of the whole row, w8a8.py:106-115)
// before it quantises its part of the row, and the int32 partial accumulators
// (a SUM over the ranks, exact) before the dequant + residual epilogue
// (w8a8.py:118-139, lightweight_runner.py:539-552). With NCCL that is
// row_absmax -> all-reduce(MAX) -> quantise -> linear -> all-reduce(SUM) ->
// dequant. Here each exchange is one kernel that also does the work next to
// it:
//
//   npl_tp_absmax_quant     local row absmax, pushed to every peer; the whole
//                           row's max; the row quantised with it
//   npl_tp_allreduce_dequant the local partial accumulators pushed to every
//                           peer; the sum of all ranks' partials; dequant
//                           (+ residual) to fp16
//
// Every rank maps every other rank's exchange buffer (CUDA IPC, npl_ipc_*),
// so a push is a plain store into the peer's HBM over NVLink, followed by a
// release store of a per-slice sequence number into the peer's flag word.
// The receiver waits (bounded, ~1 s) until the flag of every peer reaches its
// own sequence number, then reads the pushed data from its own memory. The
// sequence numbers live in device memory (each CTA keeps the count of calls
// it has made), so the kernels need nothing from the host per call and can
// be captured in a CUDA graph. The data slots alternate between two halves by
// call parity: a rank can be at most one call ahead of a peer (it cannot pass
// call n + 1 before every peer has started it, which needs the peer's call n
// to have finished), so a slot is never overwritten while it is being read.
// No TMA and no bulk copies: only plain loads and stores.
#include <algorithm>
#include <cstring>

#include "npl_common.cuh"

namespace npl {
namespace {

constexpr int kXMaxRanks = 8;
constexpr int kXSumCtas = 64;    // slices of the accumulator exchange (fixed, so call counts line up)
constexpr int kXMaxRows = 64;    // tokens per call (decode batches)
constexpr int kXThreads = 256;

struct XLayout {
  size_t flags_sum, flags_max, seen_sum, seen_max, data_sum, data_max, total;
};

XLayout x_layout(int world, long long max_elems) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  XLayout l;
  l.flags_sum = 0;
  l.flags_max = l.flags_sum + al(sizeof(uint32_t) * kXMaxRanks * kXSumCtas);
  l.seen_sum = l.flags_max + al(sizeof(uint32_t) * kXMaxRanks * kXMaxRows);
  l.seen_max = l.seen_sum + al(sizeof(uint32_t) * kXSumCtas);
  l.data_sum = l.seen_max + al(sizeof(uint32_t) * kXMaxRows);
  l.data_max = l.data_sum + al(sizeof(int32_t) * 2 * (size_t)world * (size_t)max_elems);
  l.total = l.data_max + al(sizeof(int32_t) * 2 * (size_t)world * kXMaxRows);
  return l;
}

struct XArgs {
  int world, rank;
  char* buf[kXMaxRanks];  // every rank's exchange buffer, as mapped in this process
  long long max_elems;
  XLayout lay;
  int* status;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Thread 0: after every thread's pushes (each thread fenced its own stores at
// system scope, then the CTA met at a barrier), raise this slice's flag in
// every peer to `seq`, then wait until every peer has raised ours. Returns
// false (and records the code) when a peer did not arrive within ~1 s.
__device__ bool exchange_flags(const XArgs& a, size_t flags_off, int slots, int slot, uint32_t seq) {
  for (int p = 0; p < a.world; ++p)
    if (p != a.rank)
      st_release_sys(reinterpret_cast<uint32_t*>(a.buf[p] + flags_off) + (size_t)a.rank * slots + slot, seq);
  const uint32_t* own = reinterpret_cast<const uint32_t*>(a.buf[a.rank] + flags_off);
  for (int q = 0; q < a.world; ++q) {
    if (q == a.rank) continue;
    const uint32_t* f = own + (size_t)q * slots + slot;
    if ((int32_t)(ld_acquire_sys(f) - seq) >= 0) continue;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(f) - seq) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (a.status) atomicCAS(a.status, 0, NPL_DEV_TIMEOUT_PEER);
        return false;
      }
    }
  }
  __threadfence();
  return true;
}

__device__ __forceinline__ void load_h8(const __half* p, float (&v)[8]) {
  const uint4 x = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// One CTA per token row m: max |x[m, :K]| of this rank's part, pushed to every
// peer; the max over all ranks; the row quantised with it exactly as
// npl_quant_rows (w8a8.py:33-50).
__global__ void __launch_bounds__(kXThreads) xchg_absmax_quant_kernel(XArgs a, const __half* __restrict__ x, int K,
                                                                      int ldx, int8_t* __restrict__ q, int ldq,
                                                                      float* __restrict__ scale) {
  __shared__ float red[32];
  __shared__ float s_amax;
  __shared__ uint32_t s_seq;
  __shared__ int s_ok;
  const int m = blockIdx.x;
  char* own = a.buf[a.rank];
  uint32_t* seen = reinterpret_cast<uint32_t*>(own + a.lay.seen_max) + m;
  pdl_wait();
  if (threadIdx.x == 0) s_seq = *seen + 1;
  const __half* row = x + (size_t)m * ldx;
  float amax = 0.f;
  for (int c = threadIdx.x * 8; c < K; c += kXThreads * 8) {
    float v[8];
    load_h8(row + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = block_max(amax, red);  // its barriers also publish s_seq
  const uint32_t seq = s_seq;
  const int par = (int)(seq & 1u);
  if (threadIdx.x == 0) {
    for (int p = 0; p < a.world; ++p)
      if (p != a.rank)
        reinterpret_cast<int32_t*>(a.buf[p] + a.lay.data_max)[((size_t)par * a.world + a.rank) * kXMaxRows + m] =
            __float_as_int(amax);
    __threadfence_system();
    s_ok = exchange_flags(a, a.lay.flags_max, kXMaxRows, m, seq);
    if (s_ok) {
      const int32_t* d = reinterpret_cast<const int32_t*>(own + a.lay.data_max);
      for (int p = 0; p < a.world; ++p)
        if (p != a.rank) amax = fmaxf(amax, __int_as_float(__ldcg(d + ((size_t)par * a.world + p) * kXMaxRows + m)));
      s_amax = amax;
    }
  }
  __syncthreads();
  if (s_ok) amax = s_amax;
  const float s = scale_from_absmax(amax);
  const float rs = quant_recip(s);
  if (threadIdx.x == 0) {
    scale[m] = s;
    *seen = seq;
  }
  int8_t* qrow = q + (size_t)m * ldq;
  for (int c = threadIdx.x * 8; c < K; c += kXThreads * 8) {
    float v[8];
    load_h8(row + c, v);
    uint2 u;
    u.x = u.y = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = (uint32_t)(quantize_one(v[i], s, rs) & 0xff);
      if (i < 4) u.x |= b << (8 * i);
      else u.y |= b << (8 * (i - 4));
    }
    *reinterpret_cast<uint2*>(qrow + c) = u;
  }
  pdl_trigger();
}

// kXSumCtas CTAs, each one slice of the M x N accumulators (4-element units):
// the slice of this rank's partials pushed to every peer, then the sum over
// the ranks (exact int32) dequantised as npl_dequant: v = ((acc * sa[m]) *
// sw[n]) (+ bias[n]); out = fp16(v), or fp16(fp16(v) + residual[m, n]).
__global__ void __launch_bounds__(kXThreads)
    xchg_sum_dequant_kernel(XArgs a, const int32_t* __restrict__ acc, int M, int N, const float* __restrict__ sa,
                            const float* __restrict__ sw, const float* __restrict__ bias,
                            const __half* __restrict__ residual, int ld_res, __half* __restrict__ out, int ld_out) {
  __shared__ uint32_t s_seq;
  __shared__ int s_ok;
  const int j = blockIdx.x;
  char* own = a.buf[a.rank];
  uint32_t* seen = reinterpret_cast<uint32_t*>(own + a.lay.seen_sum) + j;
  const long long units = (long long)M * N / 4;
  const long long u0 = j * units / kXSumCtas, u1 = (j + 1) * units / kXSumCtas;
  pdl_wait();
  if (threadIdx.x == 0) s_seq = *seen + 1;
  __syncthreads();
  const uint32_t seq = s_seq;
  const int par = (int)(seq & 1u);
  const int4* mine = reinterpret_cast<const int4*>(acc);
  for (int p = 0; p < a.world; ++p) {
    if (p == a.rank) continue;
    int4* dst = reinterpret_cast<int4*>(a.buf[p] + a.lay.data_sum) +
                ((size_t)par * a.world + a.rank) * (size_t)(a.max_elems / 4);
    for (long long u = u0 + threadIdx.x; u < u1; u += kXThreads) dst[u] = mine[u];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_ok = exchange_flags(a, a.lay.flags_sum, kXSumCtas, j, seq);
  __syncthreads();
  if (threadIdx.x == 0) *seen = seq;
  if (!s_ok) return;  // status recorded; the output is not written
  const int4* recv = reinterpret_cast<const int4*>(own + a.lay.data_sum);
  for (long long u = u0 + threadIdx.x; u < u1; u += kXThreads) {
    int4 v = mine[u];
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) continue;
      const int4 w = __ldcg(recv + ((size_t)par * a.world + p) * (size_t)(a.max_elems / 4) + u);
      v.x += w.x;
      v.y += w.y;
      v.z += w.z;
      v.w += w.w;
    }
    const long long e = u * 4;
    const int m = (int)(e / N), n = (int)(e % N);
    const int32_t iv[4] = {v.x, v.y, v.z, v.w};
    __half o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f = __fmul_rn(__fmul_rn(__int2float_rn(iv[i]), sa[m]), sw[n + i]);
      if (bias) f = __fadd_rn(f, bias[n + i]);
      if (residual) {
        const float r = __half2float(residual[(size_t)m * ld_res + n + i]);
        o[i] = __float2half_rn(__fadd_rn(__half2float(__float2half_rn(f)), r));
      } else {
        o[i] = __float2half_rn(f);
      }
    }
    __half* dst = out + (size_t)m * ld_out + n;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = o[i];
  }
  pdl_trigger();
}

int make_xargs(const npl_tp_peers* peers, XArgs* a, const char* what) {
  if (!peers) return fail(NPL_ERR_ARG, "%s: null peers", what);
  if (peers->world < 1 || peers->world > kXMaxRanks || peers->rank < 0 || peers->rank >= peers->world ||
      peers->max_elems <= 0 || peers->max_elems % 4)
    return fail(NPL_ERR_ARG, "%s: bad peers (world %d, rank %d, max_elems %lld)", what, peers->world, peers->rank,
                peers->max_elems);
  a->world = peers->world;
  a->rank = peers->rank;
  for (int r = 0; r < kXMaxRanks; ++r) {
    a->buf[r] = r < peers->world ? static_cast<char*>(peers->buffers[r]) : nullptr;
    if (r < peers->world && (!a->buf[r] || (reinterpret_cast<uintptr_t>(a->buf[r]) & 255u)))
      return fail(NPL_ERR_ARG, "%s: exchange buffer of rank %d is null or not 256-byte aligned", what, r);
  }
  a->max_elems = peers->max_elems;
  a->lay = x_layout(peers->world, peers->max_elems);
  a->status = device_status_ptr();
  return NPL_OK;
}

using PFN_getAddressRange = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

int allocation_base(const void* ptr, char** base) {
  static PFN_getAddressRange fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(NPL_ERR_LAUNCH, "cuMemGetAddressRange unavailable");
    fn = reinterpret_cast<PFN_getAddressRange>(f);
  }
  CUdeviceptr b = 0;
  size_t size = 0;
  if (fn(&b, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(NPL_ERR_ARG, "npl_ipc_handle: not a device allocation");
  *base = reinterpret_cast<char*>(b);
  return NPL_OK;
}

}  // namespace
}  // namespace npl

using namespace npl;

extern "C" size_t npl_tp_exchange_bytes(int world, long long max_elems) {
  if (world < 1 || world > kXMaxRanks || max_elems <= 0 || max_elems % 4) return 0;
  return x_layout(world, max_elems).total;
}

extern "C" int npl_ipc_handle(const void* ptr, void* handle_out, size_t* offset_out) {
  if (int rc = check_device()) return rc;
  if (!ptr || !handle_out || !offset_out) return fail(NPL_ERR_ARG, "npl_ipc_handle: null pointer");
  char* base = nullptr;
  if (int rc = allocation_base(ptr, &base)) return rc;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, base);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(NPL_ERR_LAUNCH, "npl_ipc_handle: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == NPL_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = (size_t)(static_cast<const char*>(ptr) - base);
  return NPL_OK;
}

extern "C" int npl_ipc_open(const void* handle, size_t offset, void** ptr_out, void** base_out) {
  if (int rc = check_device()) return rc;
  if (!handle || !ptr_out || !base_out) return fail(NPL_ERR_ARG, "npl_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(NPL_ERR_LAUNCH, "npl_ipc_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  }
  *base_out = base;
  *ptr_out = static_cast<char*>(base) + offset;
  return NPL_OK;
}

extern "C" int npl_ipc_close(void* base) {
  if (!base) return fail(NPL_ERR_ARG, "npl_ipc_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(NPL_ERR_LAUNCH, "npl_ipc_close: %s", cudaGetErrorString(e));
  }
  return NPL_OK;
}

extern "C" int npl_tp_absmax_quant(const npl_tp_peers* peers, const void* x, int M, int K, int ldx, int8_t* q,
                                   int ldq, float* scale, void* stream) {
  if (int rc = check_device()) return rc;
  XArgs a{};
  if (int rc = make_xargs(peers, &a, "npl_tp_absmax_quant")) return rc;
  if (!x || !q || !scale) return fail(NPL_ERR_ARG, "npl_tp_absmax_quant: null pointer");
  if (M < 0 || M > kXMaxRows || K <= 0 || K % 16 || ldx < K || ldx % 8 || ldq < K || ldq % 16)
    return fail(NPL_ERR_ARG, "npl_tp_absmax_quant: bad shape M=%d (<= %d) K=%d ldx=%d ldq=%d", M, kXMaxRows, K, ldx,
                ldq);
  if (!aligned16(x) || !aligned16(q)) return fail(NPL_ERR_ARG, "npl_tp_absmax_quant: pointers must be 16-B aligned");
  if (M == 0) return NPL_OK;
  return launch_pdl("npl_tp_absmax_quant", xchg_absmax_quant_kernel, dim3(M), dim3(kXThreads), 0,
                    static_cast<cudaStream_t>(stream), a, static_cast<const __half*>(x), K, ldx, q, ldq, scale);
}

extern "C" int npl_tp_allreduce_dequant(const npl_tp_peers* peers, const int32_t* acc, int M, int N, const float* sa,
                                        const float* sw, const float* bias, const void* residual, int ld_res,
                                        void* out, int ld_out, void* stream) {
  if (int rc = check_device()) return rc;
  XArgs a{};
  if (int rc = make_xargs(peers, &a, "npl_tp_allreduce_dequant")) return rc;
  if (!acc || !sa || !sw || !out) return fail(NPL_ERR_ARG, "npl_tp_allreduce_dequant: null pointer");
  if (M < 0 || N <= 0 || N % 4 || ld_out < N || ld_out % 4 || (residual && (ld_res < N || ld_res % 4)) ||
      (long long)M * N > a.max_elems)
    return fail(NPL_ERR_ARG, "npl_tp_allreduce_dequant: bad shape M=%d N=%d (M*N <= %lld, N %% 4 == 0)", M, N,
                a.max_elems);
  if (!aligned16(acc)) return fail(NPL_ERR_ARG, "npl_tp_allreduce_dequant: acc must be 16-byte aligned");
  if (M == 0) return NPL_OK;
  return launch_pdl("npl_tp_allreduce_dequant", xchg_sum_dequant_kernel, dim3(kXSumCtas), dim3(kXThreads), 0,
                    static_cast<cudaStream_t>(stream), a, acc, M, N, sa, sw, bias,
                    static_cast<const __half*>(residual), ld_res, static_cast<__half*>(out), ld_out);
}
