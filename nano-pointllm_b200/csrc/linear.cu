// W8A8 linear on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// Replaces w8a8.py:118-139 (integer_linear_per_output_reference) and the
// F.linear projection call sites of the decode/prefill path (packed QKV, O,
// packed gate/up + act_fn(gate) * up, down, LM head).
//
// Formulation ("swap AB"): the weight tile is the MMA's A operand and the
// tokens are its N dimension,
//     D[n, m] = sum_k W[n, k] * X[m, k]      (A = W: 128 rows, B = X: NT rows)
// so a decode batch of M <= 64 tokens fills an MMA of 128 x NT x 32 with
// NT = 8..64, and prefill uses NT = 128/256 token tiles.
//
// Per CTA (192 threads, one CTA per SM):
//   warp 0     TMA producer: W tile [128 rows x 128 B] + X tile [NT x 128 B]
//              per stage, 128-byte swizzle, STAGES-deep ring in shared memory
//   warp 1     TMEM owner + MMA issuer (one thread): 4 MMAs of K = 32 per
//              stage into a double-buffered int32 accumulator in TMEM
//   warps 2-5  epilogue: tcgen05.ld (TMEM lane = weight row, column = token),
//              dequant ((acc * sa) * sw + bias), fused residual / SiLU*up,
//              fp16 or fp32 stores
//
// Work split ("stream-K"): the (tile, k-block) units of the whole problem are
// divided evenly over the grid. A CTA that owns a whole tile runs its
// epilogue from TMEM; partial tiles are reduced through int32 atomics in the
// caller's workspace (exact and order-independent), and the CTA whose
// k-blocks complete the count runs the epilogue and clears the workspace.
// Only a tile cut by a CTA boundary is partial, so the workspace holds
// grid - 1 tile slots; a partial tile uses the slot of the first boundary
// inside it.
//
// All mbarrier waits are bounded (~1 s); on expiry the kernel records a code
// in the device status word, drains its in-flight copies and MMAs, frees TMEM
// and returns.
#include <cudaTypedefs.h>

#include <algorithm>
#include <initializer_list>

#include "npl_common.cuh"

namespace npl {
namespace {

constexpr int kTileN = 128;   // weight rows per tile (MMA M)
constexpr int kBlockK = 128;  // K bytes per stage (one 128-byte swizzle atom)
constexpr int kThreads = 192;

struct LinearArgs {
  int M, N, K;
  const float* sa;
  const float* sw;
  const float* bias;
  int epilogue;
  const __half* residual;
  int ld_res;
  void* out;
  int ld_out;
  int out_dtype;
  int32_t* acc_out;
  int32_t* ws_acc;  // [grid - 1 slots][NT][128]
  int32_t* ws_cnt;  // [grid - 1 slots]
  int n_tiles;
  int k_blocks;
  long long total_units;
  int* status;
};

template <int NT, int STAGES>
struct alignas(1024) LinearSmem {
  int8_t a[STAGES][kTileN * kBlockK];
  int8_t b[STAGES][NT * kBlockK];
  __half xchg[8][64];  // SiLU*up: up values of one 8-column chunk
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t teardown;
  uint32_t tmem_base;
  int last_flag;
};

__host__ __device__ constexpr uint32_t tmem_cols_for(int nt) {
  uint32_t c = 32;
  while (c < 2u * (uint32_t)nt) c <<= 1;
  return c;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Iterates the CTA's stream-K segments: (tile, kb0, kb1).
struct SegmentIter {
  long long u, u1;
  int k_blocks;
  __device__ SegmentIter(const LinearArgs& p) {
    u = (long long)blockIdx.x * p.total_units / gridDim.x;
    u1 = (long long)(blockIdx.x + 1) * p.total_units / gridDim.x;
    k_blocks = p.k_blocks;
  }
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (u >= u1) return false;
    tile = (int)(u / k_blocks);
    kb0 = (int)(u % k_blocks);
    kb1 = (int)min((long long)k_blocks, kb0 + (u1 - u));
    u += kb1 - kb0;
    return true;
  }
};

__device__ __forceinline__ float dequant(int32_t acc, float sa, float sw, const float* bias, int n) {
  float v = __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw);
  if (bias) v = __fadd_rn(v, bias[n]);
  return v;
}

// silu(g) rounded once to fp16, evaluated in fp64.
__device__ __forceinline__ float silu_h(float g) {
  const double gd = (double)g;
  return __half2float(__double2half(gd / (1.0 + exp(-gd))));
}

// Epilogue of 8 consecutive token columns [c0, c0 + 8) of tile row `row`.
template <int NT>
__device__ __forceinline__ void epilogue_chunk(const LinearArgs& p, __half (*xchg)[64], int m_tile, int n_tile,
                                               int row, int c0, const int32_t (&acc)[8]) {
  const int n = n_tile * kTileN + row;
  const int m_base = m_tile * NT + c0;
  if (p.acc_out && n < p.N) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (m_base + j < p.M) p.acc_out[(size_t)(m_base + j) * p.N + n] = acc[j];
  }
  if (p.epilogue == NPL_EPI_SILU_MUL) {
    // rows 0-63 gate, 64-127 up of output columns n_tile*64 + (row % 64)
    const float sw = p.sw[n];
    if (row >= 64) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = min(m_base + j, p.M - 1);
        xchg[j][row - 64] = __float2half_rn(dequant(acc[j], p.sa[m], sw, p.bias, n));
      }
    }
    epi_bar();
    if (row < 64) {
      const int col = n_tile * 64 + row;
      __half* out = static_cast<__half*>(p.out);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = m_base + j;
        if (m < p.M) {
          const float g = __half2float(__float2half_rn(dequant(acc[j], p.sa[m], sw, p.bias, n)));
          const float u = __half2float(xchg[j][row]);
          out[(size_t)m * p.ld_out + col] = __float2half_rn(__fmul_rn(silu_h(g), u));
        }
      }
    }
    epi_bar();
    return;
  }
  if (n >= p.N) return;
  const float sw = p.sw[n];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int m = m_base + j;
    if (m >= p.M) break;
    const float v = dequant(acc[j], p.sa[m], sw, p.bias, n);
    if (p.epilogue == NPL_EPI_RESIDUAL) {
      const float o = __half2float(__float2half_rn(v));
      const float r = __half2float(p.residual[(size_t)m * p.ld_res + n]);
      static_cast<__half*>(p.out)[(size_t)m * p.ld_out + n] = __float2half_rn(__fadd_rn(o, r));
    } else if (p.out_dtype == NPL_F32) {
      static_cast<float*>(p.out)[(size_t)m * p.ld_out + n] = v;
    } else {
      static_cast<__half*>(p.out)[(size_t)m * p.ld_out + n] = __float2half_rn(v);
    }
  }
}

template <int NT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    w8a8_linear_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                       const LinearArgs p) {
  extern __shared__ unsigned char smem_raw[];
  using Smem = LinearSmem<NT, STAGES>;
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr uint32_t kTmemCols = tmem_cols_for(NT);
  constexpr uint32_t kStageBytes = kTileN * kBlockK + NT * kBlockK;
  constexpr uint32_t kIdesc = idesc_i8(kTileN, NT);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmap_w);
    prefetch_tensormap(&tmap_x);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], 4);
    }
    mbar_init(&s.teardown, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = s.tmem_base;
  pdl_trigger();  // the next kernel may start launching its CTAs

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      // Weights do not depend on earlier kernels: the weight tiles of the
      // first ring stages are requested before waiting for the previous
      // kernel; the token tiles (its output) only after.
      int pre = 0;
      {
        SegmentIter it(p);
        int tile, kb0, kb1;
        while (pre < STAGES && it.next(tile, kb0, kb1)) {
          const int n_tile = tile % p.n_tiles;
          for (int kb = kb0; kb < kb1 && pre < STAGES; ++kb, ++pre) {
            mbar_arrive_expect_tx(&s.full[pre], kStageBytes);
            tma_load_2d(s.a[pre], &tmap_w, kb * kBlockK, n_tile * kTileN, &s.full[pre], pol_w);
          }
        }
      }
      uint32_t outstanding = pre >= 32 ? 0xffffffffu : ((1u << pre) - 1);  // stages holding a load
      pdl_wait();
      SegmentIter it(p);
      int tile, kb0, kb1, stage = 0, unit = 0;
      uint32_t phase = 0;
      bool ok = true;
      while (ok && it.next(tile, kb0, kb1)) {
        const int m_tile = tile / p.n_tiles, n_tile = tile % p.n_tiles;
        for (int kb = kb0; kb < kb1; ++kb, ++unit) {
          if (unit >= pre) {
            if (!mbar_wait(&s.empty[stage], phase ^ 1, p.status, NPL_DEV_TIMEOUT_TMA)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&s.full[stage], kStageBytes);
            tma_load_2d(s.a[stage], &tmap_w, kb * kBlockK, n_tile * kTileN, &s.full[stage], pol_w);
          }
          tma_load_2d(s.b[stage], &tmap_x, kb * kBlockK, m_tile * NT, &s.full[stage], pol_x);
          outstanding |= 1u << stage;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }

      // Drain: every issued load must land before the CTA's shared memory is
      // released. A stage's last load used parity (phase of that issue).
      for (int i = 0; i < STAGES; ++i) {
        if (!(outstanding >> i & 1)) continue;
        // stages before `stage` were last issued in the current phase, the
        // others in the previous one
        const uint32_t par = i < stage ? phase : phase ^ 1;
        mbar_wait(&s.full[i], par, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      SegmentIter it(p);
      int tile, kb0, kb1, stage = 0, seg = 0;
      uint32_t phase = 0;
      bool ok = true;
      while (ok && it.next(tile, kb0, kb1)) {
        const int buf = seg & 1;
        const uint32_t tphase = (seg >> 1) & 1;
        if (!mbar_wait(&s.tempty[buf], tphase ^ 1, p.status, NPL_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * NT);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&s.full[stage], phase, p.status, NPL_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(s.a[stage]);
          const uint32_t b0 = smem_u32(s.b[stage]);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 32; ++kk) {
            mma_i8(d, sdesc_k_sw128(a0 + kk * 32), sdesc_k_sw128(b0 + kk * 32), kIdesc,
                   (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&s.empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&s.tfull[buf]);
        ++seg;
      }
      // all MMAs issued by this thread complete before TMEM is freed
      tc_commit(&s.teardown);
      mbar_wait(&s.teardown, 0, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;
    pdl_wait();
    SegmentIter it(p);
    int tile, kb0, kb1, seg = 0;
    while (it.next(tile, kb0, kb1)) {
      const int buf = seg & 1;
      const uint32_t tphase = (seg >> 1) & 1;
      const int m_tile = tile / p.n_tiles, n_tile = tile % p.n_tiles;
      if (!mbar_wait(&s.tfull[buf], tphase, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * NT);
      const bool whole = (kb0 == 0 && kb1 == p.k_blocks);
      // slot = (first CTA boundary strictly inside the tile) - 1
      const long long first_unit = (long long)tile * p.k_blocks;
      const int slot = (int)(((first_unit + 1) * gridDim.x + p.total_units - 1) / p.total_units) - 1;
      int32_t* ws = p.ws_acc + (size_t)slot * NT * kTileN;
      if (whole) {
        for (int c0 = 0; c0 < NT; c0 += 8) {
          int32_t acc[8];
          tmem_ld_x8(taddr + c0, acc);
          tmem_wait_ld();
          epilogue_chunk<NT>(p, s.xchg, m_tile, n_tile, row, c0, acc);
        }
      } else {
        for (int c0 = 0; c0 < NT; c0 += 8) {
          int32_t acc[8];
          tmem_ld_x8(taddr + c0, acc);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (m_tile * NT + c0 + j < p.M) atomicAdd(ws + (size_t)(c0 + j) * kTileN + row, acc[j]);
        }
      }
      // accumulator buffer free for the next segment's MMAs
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.tempty[buf]);
      if (!whole) {
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const int prev = atomicAdd(p.ws_cnt + slot, kb1 - kb0);
          s.last_flag = (prev + (kb1 - kb0) == p.k_blocks);
        }
        epi_bar();
        if (s.last_flag) {
          __threadfence();
          for (int c0 = 0; c0 < NT; c0 += 8) {
            int32_t acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              int32_t* cell = ws + (size_t)(c0 + j) * kTileN + row;
              acc[j] = __ldcg(cell);
              __stcg(cell, 0);
            }
            epilogue_chunk<NT>(p, s.xchg, m_tile, n_tile, row, c0, acc);
          }
          if (threadIdx.x == 64) p.ws_cnt[slot] = 0;
        }
        epi_bar();
      }
      ++seg;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// int8 row-major [rows, cols] with row stride ld bytes; box [box_rows, 128 B].
int make_map(CUtensorMap* map, const void* base, int rows, int cols, int ld, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(NPL_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld};
  const cuuint32_t box[2] = {(cuuint32_t)kBlockK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NPL_ERR_ARG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NPL_OK;
}

int pick_nt(int M) {
  if (M <= 8) return 8;
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  return 256;
}

// Workspace: grid - 1 partial-tile slots of NT x 128 int32 plus one counter
// per slot; grid <= number of SMs of the current device.
int max_grid() {
  const int sms = num_sms();
  return sms > 0 ? sms : 148;
}

size_t ws_acc_bytes(int M) {
  const size_t slots = (size_t)std::max(1, max_grid() - 1);
  return slots * pick_nt(M) * kTileN * sizeof(int32_t);
}

size_t ws_bytes(int M) {
  const size_t slots = (size_t)std::max(1, max_grid() - 1);
  return ws_acc_bytes(M) + ((slots * sizeof(int32_t) + 255) & ~size_t(255));
}

template <int NT, int STAGES>
int launch_linear(const CUtensorMap& tw, const CUtensorMap& tx, LinearArgs& p, cudaStream_t st) {
  auto kern = w8a8_linear_kernel<NT, STAGES>;
  const int smem = (int)sizeof(LinearSmem<NT, STAGES>) + 1024;
  static bool configured = false;  // per instantiation; attribute is per device function
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return launch_status("npl_w8a8_linear: smem attribute");
    configured = true;
  }
  const long long grid = std::min<long long>(max_grid(), p.total_units);
  return launch_pdl("npl_w8a8_linear", kern, dim3((unsigned)grid), dim3(kThreads), (size_t)smem, st, tw, tx, p);
}

}  // namespace
}  // namespace npl

using namespace npl;

extern "C" size_t npl_linear_workspace_bytes(int M, int N, int K) {
  (void)K;
  if (M <= 0 || N <= 0) return 0;
  return ws_bytes(M);
}

extern "C" int npl_w8a8_linear(const int8_t* qa, int lda, const float* sa, const int8_t* qw, int ldw,
                               const float* sw, const float* bias, int M, int N, int K, int epilogue,
                               const void* residual, int ld_res, void* out, int ld_out, int out_dtype,
                               int32_t* acc_out, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_device()) return rc;
  if (!qa || !sa || !qw || !sw || !out) return fail(NPL_ERR_ARG, "npl_w8a8_linear: null pointer");
  if (M < 0 || N <= 0 || K <= 0 || K % 16 || lda < K || lda % 16 || ldw < K || ldw % 16)
    return fail(NPL_ERR_ARG, "npl_w8a8_linear: bad shape M=%d N=%d K=%d lda=%d ldw=%d", M, N, K, lda, ldw);
  if ((long long)K * 127 * 127 >= (1ll << 31))
    return fail(NPL_ERR_OVERFLOW, "npl_w8a8_linear: worst-case dot product exceeds signed INT32 (K=%d)", K);
  if (!aligned16(qa) || !aligned16(qw)) return fail(NPL_ERR_ARG, "npl_w8a8_linear: int8 operands must be 16-byte aligned");
  if (epilogue == NPL_EPI_RESIDUAL) {
    if (!residual || out_dtype != NPL_F16 || ld_res < N || ld_out < N)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: residual epilogue needs fp16 residual/out with ld >= N");
  } else if (epilogue == NPL_EPI_SILU_MUL) {
    if (N % kTileN || out_dtype != NPL_F16 || ld_out < N / 2)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: SiLU*up epilogue needs N %% 128 == 0, fp16 out, ld_out >= N/2");
  } else if (epilogue == NPL_EPI_NONE) {
    if ((out_dtype != NPL_F16 && out_dtype != NPL_F32) || ld_out < N)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: out_dtype must be NPL_F16/NPL_F32 and ld_out >= N");
  } else {
    return fail(NPL_ERR_ARG, "npl_w8a8_linear: unknown epilogue %d", epilogue);
  }
  if (M == 0) return NPL_OK;
  const size_t need = ws_bytes(M);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(NPL_ERR_ARG, "npl_w8a8_linear: workspace of %zu bytes (16-byte aligned) required", need);

  const int nt = pick_nt(M);
  LinearArgs p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.sa = sa;
  p.sw = sw;
  p.bias = bias;
  p.epilogue = epilogue;
  p.residual = static_cast<const __half*>(residual);
  p.ld_res = ld_res;
  p.out = out;
  p.ld_out = ld_out;
  p.out_dtype = out_dtype;
  p.acc_out = acc_out;
  p.ws_acc = static_cast<int32_t*>(workspace);
  p.ws_cnt = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + ws_acc_bytes(M));
  p.n_tiles = (N + kTileN - 1) / kTileN;
  p.k_blocks = (K + kBlockK - 1) / kBlockK;
  const int m_tiles = (M + nt - 1) / nt;
  p.total_units = (long long)p.n_tiles * m_tiles * p.k_blocks;
  p.status = device_status_ptr();

  CUtensorMap tw, tx;
  if (int rc = make_map(&tw, qw, N, K, ldw, kTileN)) return rc;
  if (int rc = make_map(&tx, qa, M, K, lda, nt)) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Decode tiles (NT <= 64) keep the ring near 100 KB so that the next
  // kernel's CTA fits beside this one on an SM and starts its weight loads
  // while this one finishes (programmatic dependent launch).
  switch (nt) {
    case 8: return launch_linear<8, 6>(tw, tx, p, st);
    case 16: return launch_linear<16, 6>(tw, tx, p, st);
    case 32: return launch_linear<32, 5>(tw, tx, p, st);
    case 64: return launch_linear<64, 4>(tw, tx, p, st);
    case 128: return launch_linear<128, 6>(tw, tx, p, st);
    default: return launch_linear<256, 4>(tw, tx, p, st);
  }
}

// ----------------------------------------------------------------------------
// npl_w8a8_linear_noalloc: the same linear for callers that cannot allocate.
//
// npl_w8a8_linear needs a caller-provided workspace for the partial tiles of
// its stream-K split. Some callers cannot provide one: a plugin running inside
// a host engine that owns every byte of device memory and hands the plugin
// only its input and output buffers, a binding from a language that has no
// CUDA allocator, or a latency-critical loop that must not call cudaMalloc
// (which may synchronise the device). For them this entry point takes its
// scratch from a fixed array in the library's own device memory instead.
//
// The array below is sized for at most 64 tokens (M <= 64) on a device with
// at most 160 SMs: 159 partial-tile slots of 64 x 128 int32 plus their
// counters, about 5 MiB. It exists once per device that loads the library and
// stays allocated until the process exits. Every call uses the same array, so
// calls must not overlap on the GPU: two calls in flight at the same time (on
// different streams, or in different host threads) race on it and give wrong
// results. Each call zeroes the part it uses (on the caller's stream) before
// the kernel runs, so a call never depends on what an earlier call left there.
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress (with that device current); make that first call
// before starting any stream capture.
// ----------------------------------------------------------------------------
namespace npl {
namespace {

constexpr int kNoAllocMaxTokens = 64;
constexpr int kNoAllocMaxSlots = 159;  // grid - 1 for devices with up to 160 SMs
constexpr size_t kNoAllocAccBytes = (size_t)kNoAllocMaxSlots * kNoAllocMaxTokens * kTileN * sizeof(int32_t);
constexpr size_t kNoAllocBytes = kNoAllocAccBytes + ((kNoAllocMaxSlots * sizeof(int32_t) + 255) & ~size_t(255));

static __device__ __align__(256) unsigned char g_linear_scratch[kNoAllocBytes];

constexpr int kNoAllocDevices = 64;
void* g_scratch_ptr[kNoAllocDevices];

// Device address of g_linear_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocDevices)
    return fail(NPL_ERR_LAUNCH, "npl_w8a8_linear_noalloc: no usable current device");
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (e != cudaSuccess || !p)
      return fail(NPL_ERR_LAUNCH, "npl_w8a8_linear_noalloc: cudaGetSymbolAddress failed: %s",
                  cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return NPL_OK;
}

}  // namespace
}  // namespace npl

extern "C" int npl_w8a8_linear_noalloc(const int8_t* qa, int lda, const float* sa, const int8_t* qw, int ldw,
                                       const float* sw, const float* bias, int M, int N, int K, int epilogue,
                                       const void* residual, int ld_res, void* out, int ld_out, int out_dtype,
                                       int32_t* acc_out, void* stream) {
  if (int rc = check_device()) return rc;
  if (M > npl::kNoAllocMaxTokens)
    return fail(NPL_ERR_ARG, "npl_w8a8_linear_noalloc: M = %d tokens, the built-in scratch holds at most %d", M,
                npl::kNoAllocMaxTokens);
  if (M <= 0 || N <= 0 || K <= 0) {
    // shape errors (and M == 0) are reported by npl_w8a8_linear itself
    return npl_w8a8_linear(qa, lda, sa, qw, ldw, sw, bias, M, N, K, epilogue, residual, ld_res, out, ld_out,
                           out_dtype, acc_out, nullptr, 0, stream);
  }
  const size_t need = ws_bytes(M);
  if (need > npl::kNoAllocBytes)
    return fail(NPL_ERR_UNSUPPORTED,
                "npl_w8a8_linear_noalloc: this device needs %zu scratch bytes, the built-in array has %zu "
                "(more than %d SMs)",
                need, npl::kNoAllocBytes, npl::kNoAllocMaxSlots + 1);
  void* scratch = nullptr;
  if (int rc = npl::scratch_address(&scratch)) return rc;
  if (cudaMemsetAsync(scratch, 0, need, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return launch_status("npl_w8a8_linear_noalloc: clearing the scratch");
  return npl_w8a8_linear(qa, lda, sa, qw, ldw, sw, bias, M, N, K, epilogue, residual, ld_res, out, ld_out,
                         out_dtype, acc_out, scratch, need, stream);
}
