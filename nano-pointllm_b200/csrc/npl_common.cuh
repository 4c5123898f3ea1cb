// Shared device/host helpers for libnpl_w8a8 (sm_100a only).
//
// Numerics rule for every kernel of the W8A8 contract: fp32 steps that must
// match the reference bit for bit use the explicit round-to-nearest intrinsics
// (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn), so the compiler cannot fuse
// them into FMAs; the library is built without --use_fast_math.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/npl_w8a8.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ != 1000)
#error "libnpl_w8a8 targets sm_100a only"
#endif

namespace npl {

// ---------------------------------------------------------------- host side
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int launch_status(const char* what);   // maps cudaGetLastError to NPL_ERR_LAUNCH
int num_sms();                         // cached per current device
int* device_status_ptr();              // address of the per-device error word
int check_device();                    // NPL_OK on an sm_100 device

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch with programmatic dependent launch (PDL): the kernel may start while
// the previous kernel on the stream is finishing; it must execute pdl_wait()
// before touching any global memory the previous kernels read or write
// (constant weights excepted), and calls pdl_trigger() to let the next kernel
// start early in turn.
// `cluster_x` > 1 launches thread-block clusters of that many consecutive
// CTAs along x (grid.x must be a multiple of it).
template <typename... KArgs, typename... Args>
int launch_pdl_cluster(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(NPL_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  }
  return NPL_OK;
}

template <typename... KArgs, typename... Args>
int launch_pdl(const char* what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
  return launch_pdl_cluster(what, kernel, grid, block, smem, st, 1u, static_cast<Args&&>(args)...);
}

// ------------------------------------------------------------- device side
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// The linear kernels read their weights before pdl_wait(): weights must not
// be written by a kernel that may still be running. npl_quant_rows, which
// quantises weights, therefore lets the next kernel launch only after its own
// writes are visible: every thread of the CTA calls this after its last
// global write (no thread may have exited early unless the whole CTA did).
__device__ __forceinline__ void pdl_trigger_after_writes() {
  __threadfence();
  __syncthreads();
  pdl_trigger();
}

// Error word shared by all kernels of the library on this device. A kernel
// that gives up a bounded wait stores its NPL_DEV_* code here; the host reads
// it with npl_device_status().
enum DeviceError : int {
  NPL_DEV_OK = 0,
  NPL_DEV_TIMEOUT_TMA = 1,
  NPL_DEV_TIMEOUT_MMA = 2,
  NPL_DEV_TIMEOUT_EPILOGUE = 3,
  NPL_DEV_TIMEOUT_TEARDOWN = 4,
  NPL_DEV_BAD_INDEX = 5,  // a slot, block-table entry or position outside its table
  NPL_DEV_TIMEOUT_PEER = 6,  // a tensor-parallel peer did not raise its exchange flag
};

constexpr float kFp16Tiny = 6.103515625e-05f;  // torch.finfo(torch.float16).tiny = 2^-14

// scale_from_absmax (w8a8.py:46-50): fp32(fp16(max(absmax, tiny) / 127)), >= tiny.
__device__ __forceinline__ float scale_from_absmax(float absmax) {
  const float raw = __fdiv_rn(fmaxf(absmax, kFp16Tiny), 127.0f);
  return fmaxf(__half2float(__float2half_rn(raw)), kFp16Tiny);
}

// quantize_symmetric (w8a8.py:33-43): clamp(rint(v / s), -127, 127), with
// v / s the correctly rounded fp32 quotient.
//
// The quotient comes from the reciprocal r = RN(1/s) (quant_recip, once per
// row) by Markstein's FMA division step (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990): q1 = RN(v r); e = v - q1 s, exact with an FMA;
// q = RN(q1 + e r), which is RN(v / s) when v, s and e are normal numbers.
// They are whenever the result can differ from 0: s >= 2^-14 is normal, and
// |v / s| >= 1/2 makes |v| >= 2^-15 and |e| >= ulp(q1 s) / 2 >= 2^-40; for
// |v / s| < 1/2 the rounded integer is 0 either way (q stays below 1/2 or
// rounds to it, and rint(+-1/2) = 0). The tests check every finite fp16 v
// against IEEE division at every scale the quantiser can produce (the 23377
// fp16 values from 2^-14 to 516), exhaustively, and fp32 v by sampling.
__device__ __forceinline__ float quant_recip(float s) { return __frcp_rn(s); }

__device__ __forceinline__ int quantize_one(float v, float s, float r) {
  const float q1 = __fmul_rn(v, r);
  const float e = __fmaf_rn(-q1, s, v);
  const float q = __fmaf_rn(e, r, q1);
  return max(-127, min(127, __float2int_rn(q)));
}

// SiLU of an fp16 value g, rounded once to fp16 from the exact value:
// fp16(g / (1 + e^-g)), the reference's act_fn(gate) on fp16 rows
// (lightweight_runner.py:358) as the oracle states it (the fp64 formula
// rounded once). Evaluated in fp32 first: y = g / RN(1 + expf(-g)) with
// __fdividef is within 5 fp32 ulps of the exact value (expf and __fdividef
// are documented at <= 2 ulps each for these operands, the add rounds once),
// so when y - d and y + d, with d = 2^-19 |y| (>= 16 ulps), round to the same
// fp16 value, so does every value between them, the exact one included.
// Otherwise (a value within ~2^-19 of an fp16 rounding midpoint, about 0.4% of
// inputs; zeros, results below ~2^-40, g below -87 where __fdividef returns
// 0, non-finite g) the fp64 formula decides. The tests check the result
// against the fp64 evaluation for every fp16 value.
// The fp64 fallback is a call, not inlined: the epilogues that evaluate SiLU
// unroll it several times, and inlined copies of the fp64 exp overflow the
// instruction cache ("no instruction" was the top warp stall of the prefill
// gate/up launch).
static __device__ __noinline__ float silu_f16_fp64(float g) {
  const double gd = (double)g;
  return __half2float(__double2half(gd / (1.0 + exp(-gd))));
}

__device__ __forceinline__ float silu_f16(float g) {
  const float y = __fdividef(g, __fadd_rn(1.0f, expf(-g)));
  const float d = fmaxf(fabsf(y) * 0x1p-19f, 0x1p-40f);
  const __half lo = __float2half_rn(__fsub_rn(y, d)), hi = __float2half_rn(__fadd_rn(y, d));
  if (__half_as_ushort(lo) == __half_as_ushort(hi) && isfinite(g)) return __half2float(lo);
  return silu_f16_fp64(g);
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions for blockDim.x <= 1024 (multiple of 32); every thread
// receives the result. `red` is shared scratch of >= 32 elements.
template <typename T>
__device__ __forceinline__ T block_max(T v, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : red[0];
  return warp_max(v);
}

template <typename T>
__device__ __forceinline__ T block_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = lane < nw ? red[lane] : T(0);
  return warp_sum(v);
}

// Upper bound of any single wait in device code: ~1 s of wall time.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and records `code` in the
// device error word) once ~kWaitLimitNs have passed without completion.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicExch(status, code);
      return false;
    }
  }
}

// ------------------------------------------------- thread-block clusters
// Address of the same shared-memory location in CTA `rank` of the cluster
// (a shared::cluster address).
__device__ __forceinline__ uint32_t cluster_map(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }

// One arrival on an mbarrier of another CTA of the cluster, ordered after this
// thread's earlier writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// mbar_wait for phases completed by other CTAs of the cluster (acquire at
// cluster scope); bounded the same way.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicExch(status, code);
      return false;
    }
  }
}

// s32 add of a register into another CTA's shared memory (DSMEM); completion
// (4 bytes) is counted on the destination CTA's mbarrier. The source is a
// register, so the issuing CTA may exit while the add is in flight.
__device__ __forceinline__ void red_add_s32_cluster(uint32_t dst_cluster, int32_t v, uint32_t bar_cluster) {
  asm volatile(
      "red.async.relaxed.cluster.shared::cluster.mbarrier::complete_tx::bytes.add.s32 [%0], %1, [%2];" ::"r"(
          dst_cluster),
      "r"(v), "r"(bar_cluster)
      : "memory");
}

// 2-D tiled TMA load into shared memory, completion counted on `bar`.
// c0 is the innermost (contiguous) coordinate in elements, c1 the row.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later reads
// of the same bytes through the async proxy (TMA, tcgen05.mma operands).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 3-D tiled TMA load (c0 innermost, in elements), completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------ tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// MMA completion (of all previously issued tcgen05.mma of this thread) arrives
// once on `bar`.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32 (kind::i8).
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem], fp16 x fp16 -> fp32 (kind::f16).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 8 consecutive 32-bit columns; thread i of the warp gets lane
// (base lane + i), columns [col, col + 8).
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, int32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}

// 16 lanes x 8 columns (the 16x256b shape); thread i of the warp gets
// r[0], r[1] = lane (base + i / 4), columns col + 2 (i % 4) and + 1, and
// r[2], r[3] = the same columns of lane (base + 8 + i / 4).
__device__ __forceinline__ void tmem_ld_16x256b(uint32_t taddr, int32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x1.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}

// 32 lanes x 32 consecutive 32-bit columns; thread i of the warp gets lane
// (base lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 accumulator
// (c_format [4,6) = 1), a/b_format [7,10) / [10,13) = 0 (F16), A K-major,
// B K-major (bit 16 = 0) or MN-major (bit 16 = 1), N >> 3 at [17,23),
// M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool b_mn_major) {
  return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Instruction descriptor of kind::i8: signed int8 A and B, both K-major, int32
// accumulator, M rows (A) x N columns (B). Bit layout: c_format [4,6) = 2
// (S32), a_format [7,10) = 1 (INT8), b_format [10,13) = 1, a/b major bits 15/16
// = 0 (K-major), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major tile stored with the 128-byte
// swizzle (each row's 128 bytes in one 128 B line, 16 B chunks XOR (row % 8),
// 8-row atoms of 1024 B back to back): start >> 4 at [0,14), leading byte
// offset 16 B (encoded 1) at [16,30), stride byte offset 1024 B (encoded 64)
// at [32,46), descriptor version 1 at [46,48), layout SWIZZLE_128B (2) at
// [61,64). Advancing along K inside the 128 B row moves the start address.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Shared-memory matrix descriptor for an MN-major operand stored with the
// 128-byte swizzle: each K row holds 64 consecutive 16-bit MN elements in one
// 128 B line (16 B chunks XOR (row % 8)), 8 K rows form a 1024 B atom. The
// leading byte offset is the distance between 64-element MN chunks, the
// stride byte offset the distance between 8-row K groups (both encoded >> 4).
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

}  // namespace npl
