// Causal varlen attention of multi-token rows (prefill and suffix prefill)
// over the paged KV pool, on the 5th-generation tensor cores (tcgen05,
// kind::f16, fp32 accumulators in TMEM).
//
// npl_paged_prefill_attention <- paged_attention.py:1142-1207
//                                (paged_varlen_attention; kernel :1037-1139)
//
// Contract (the reference kernel's): q [total_q, H, D] fp16 (rotated); the
// rows of sequence b are q[q_offsets[b] : q_offsets[b] + q_lens[b]]; its keys
// and values are the first context_lens[b] slots of its block table in the
// fp16 pool [num_blocks, block_size, Hkv, D]; query j sits at absolute
// position context_len - q_len + j and attends to keys 0..that position.
// Scores are fp32 dot products of the fp16 rows times `scale`, masked to the
// lowest float; the softmax runs online over key tiles:
//   m' = max(m, rowmax(s));  p = exp(s - m');  alpha = exp(m - m')
//   acc = acc * alpha + fp16(p) . V  (fp32 accumulation);  l = l * alpha + sum(p)
// and out = fp16(acc / l). The probabilities are rounded to fp16 for the
// P.V product and summed unrounded into l, as the reference does. Its key
// tile is 64 (here 128), so the fp16 rounding of p, the exp and the order of
// the fp32 sums differ: results agree to fp16 rounding, not bit for bit.
//
// One CTA per (128-query tile, sequence, head), 192 threads:
//   warp 4      TMA: the Q tile once, then 128-key K and V tiles through the
//               block table (2-stage ring; pieces of gcd(block_size, 128)
//               keys, 128-byte swizzle); keys past the tile's last visible
//               key are zero-filled out-of-bounds loads;
//   warp 5      MMA issue (one thread): S_j = Q K_j^T into one of two TMEM
//               buffers, then O_{j-1} = P_{j-1} V_{j-1} (V is the MN-major B
//               operand: the cache layout as is) into one of two TMEM
//               buffers, so the tensor core works on tile j while the
//               softmax warps work on tile j-1;
//   warps 0-3   one query row per thread (= TMEM lane): row max and
//               exp of S_j, fp16 P_j into shared memory (K-major, 128-byte
//               swizzle: the A operand of P.V), then acc = acc * alpha +
//               O_{j-1} in registers, finally out = acc / l.
// TMEM: S at columns [0, 256), O at [256, 512).
#include <algorithm>
#include <cfloat>
#include <initializer_list>

#include <cudaTypedefs.h>

#include "npl_common.cuh"

namespace npl {
namespace {

constexpr int kPaTile = 128;
constexpr int kPaThreads = 192;
constexpr uint32_t kPaTmemCols = 512;
constexpr int kPaMaxQTiles = 65535;  // grid.x limit of the launch shape below

template <int D>
struct PaSmem {
  static constexpr uint32_t kHalf = kPaTile * 128;        // 128 rows x 64 fp16 (one swizzle span)
  static constexpr uint32_t kTileBytes = kPaTile * D * 2;  // Q / K / V tile
  static constexpr uint32_t kPBytes = kPaTile * kPaTile * 2;
  alignas(1024) uint8_t q[kTileBytes];
  alignas(1024) uint8_t k[2][kTileBytes];
  alignas(1024) uint8_t v[2][kTileBytes];
  alignas(1024) uint8_t p[2][kPBytes];
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2], p_full[2], p_empty[2], o_full[2], o_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
};

struct PaArgs {
  __half* out;            // [total_q, H, D]
  int ld_out;             // elements between consecutive tokens of out
  const int32_t* bt;      // [B, bt_stride]
  int bt_stride;
  int max_blocks;
  const int32_t* ctx_lens;
  const int32_t* q_lens;
  const int32_t* q_offsets;
  int H, Hkv, num_blocks, block_size, piece, total_q;
  float scale;
  int* status;
};

// mbar_wait that also gives up once another role of the CTA gave up.
__device__ __forceinline__ bool pa_wait(uint64_t* bar, uint32_t parity, int* abort, int* status, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(abort)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      *reinterpret_cast<volatile int*>(abort) = 1;
      if (status) atomicCAS(status, 0, code);
      return false;
    }
  }
}

// K or V tile j (keys [j*128, j*128+128)) of sequence b, head kvh into `dst`.
// Pieces past kv_end, or whose block-table entry is invalid, are loaded from
// row `oob` (past the pool): zero-filled.
template <int D>
__device__ __forceinline__ void load_kv_tile(uint8_t* dst, const CUtensorMap* map, const PaArgs& p,
                                             const int32_t* table, int j, int kv_end, int kvh, int oob,
                                             uint64_t* bar, uint64_t pol) {
  const int n_pieces = kPaTile / p.piece;
  for (int i = 0; i < n_pieces; ++i) {
    const int pos = j * kPaTile + i * p.piece;
    int row = oob;
    if (pos < kv_end) {
      const int logical = pos / p.block_size;
      const int blk = logical < p.max_blocks ? table[logical] : -1;
      if (blk < 0 || blk >= p.num_blocks)
        atomicCAS(p.status, 0, NPL_DEV_BAD_INDEX);
      else
        row = blk * p.block_size + pos % p.block_size;
    }
#pragma unroll
    for (int hf = 0; hf < D / 64; ++hf)
      tma_load_3d(dst + hf * PaSmem<D>::kHalf + i * p.piece * 128, map, hf * 64, kvh, row, bar, pol);
  }
}

// acc = acc * alpha + O_i (TMEM buffer i & 1, this thread's lane).
template <int D>
__device__ __forceinline__ bool pa_correct(PaSmem<D>& s, float (&acc)[D], int i, float alpha, uint32_t o_tm,
                                           int* status) {
  const int ob = i & 1;
  if (!pa_wait(&s.o_full[ob], (i >> 1) & 1, &s.abort, status, NPL_DEV_TIMEOUT_EPILOGUE)) return false;
  tc_fence_after();
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    uint32_t v[32];
    tmem_ld_x32(o_tm + ob * 128 + c * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e) acc[c * 32 + e] = fmaf(acc[c * 32 + e], alpha, __uint_as_float(v[e]));
  }
  tc_fence_before();
  mbar_arrive(&s.o_empty[ob]);
  return true;
}

template <int D>
__global__ void __launch_bounds__(kPaThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const PaArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PaSmem<D>& s = *reinterpret_cast<PaSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y, h = blockIdx.z;
  const int q0 = (gridDim.x - 1 - blockIdx.x) * kPaTile;  // longest tiles first

  pdl_wait();  // q, the pool and the metadata come from earlier work on the stream
  const int q_len = p.q_lens[b];
  if (q0 >= q_len) {
    pdl_trigger();
    return;
  }
  const int ctx = p.ctx_lens[b];
  const int q_start = p.q_offsets[b];
  if (q_start < 0 || q_start > p.total_q - q_len) {  // rows outside q / out: skip the sequence
    if (threadIdx.x == 0) atomicCAS(p.status, 0, NPL_DEV_BAD_INDEX);
    pdl_trigger();
    return;
  }
  const int prefix = ctx - q_len;
  const int rows = min(kPaTile, q_len - q0);
  const int kv_end = min(ctx, prefix + q0 + rows);  // keys some row of the tile sees
  const int n_tiles = kv_end > 0 ? (kv_end + kPaTile - 1) / kPaTile : 0;
  if (prefix < 0 || ctx > p.max_blocks * p.block_size) {
    if (threadIdx.x == 0) atomicCAS(p.status, 0, NPL_DEV_BAD_INDEX);
  }
  if (n_tiles == 0) {  // no visible key: the reference's masked loads make the output 0
    if (threadIdx.x < rows) {
      uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)(q_start + q0 + threadIdx.x) * p.ld_out + (size_t)h * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) dst[c] = make_uint4(0, 0, 0, 0);
    }
    pdl_trigger();
    return;
  }

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 128);
      mbar_init(&s.p_full[i], 128);
      mbar_init(&s.p_empty[i], 1);
      mbar_init(&s.o_full[i], 1);
      mbar_init(&s.o_empty[i], 128);
    }
    mbar_init(&s.mma_done, 1);
    s.abort = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&s.tmem_base, kPaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  pdl_trigger();

  if (warp == 4) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      prefetch_tensormap(&tmap_q);
      prefetch_tensormap(&tmap_k);
      prefetch_tensormap(&tmap_v);
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_normal();  // re-read by the other query tiles of the sequence
      const int kvh = h / (p.H / p.Hkv);
      const int oob = p.num_blocks * p.block_size;
      const int32_t* table = p.bt + (size_t)b * p.bt_stride;
      mbar_arrive_expect_tx(&s.q_full, PaSmem<D>::kTileBytes);
#pragma unroll
      for (int hf = 0; hf < D / 64; ++hf)
        tma_load_3d(s.q + hf * PaSmem<D>::kHalf, &tmap_q, hf * 64, h, q_start + q0, &s.q_full, pol_q);
      int nk = 0, nv = 0;  // K and V tiles issued
      for (int j = 0; j < n_tiles; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!pa_wait(&s.k_empty[st], ph ^ 1, &s.abort, p.status, NPL_DEV_TIMEOUT_TMA)) break;
        mbar_arrive_expect_tx(&s.k_full[st], PaSmem<D>::kTileBytes);
        load_kv_tile<D>(s.k[st], &tmap_k, p, table, j, kv_end, kvh, oob, &s.k_full[st], pol_kv);
        nk = j + 1;
        if (!pa_wait(&s.v_empty[st], ph ^ 1, &s.abort, p.status, NPL_DEV_TIMEOUT_TMA)) break;
        mbar_arrive_expect_tx(&s.v_full[st], PaSmem<D>::kTileBytes);
        load_kv_tile<D>(s.v[st], &tmap_v, p, table, j, kv_end, kvh, oob, &s.v_full[st], pol_kv);
        nv = j + 1;
      }
      // Drain: every load issued here has landed before the CTA may exit
      // (already true unless a role gave up). The last load of each stage is
      // the newest phase of its barrier.
      mbar_wait(&s.q_full, 0, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
      for (int j = max(0, nk - 2); j < nk; ++j)
        mbar_wait(&s.k_full[j & 1], (j >> 1) & 1, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
      for (int j = max(0, nv - 2); j < nv; ++j)
        mbar_wait(&s.v_full[j & 1], (j >> 1) & 1, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_f16(kPaTile, kPaTile, false);
      constexpr uint32_t kIdPV = idesc_f16(kPaTile, D, true);
      const uint32_t q_addr = smem_u32(s.q);
      auto issue_pv = [&](int i) -> bool {
        const int pb = i & 1;
        const uint32_t ph = (i >> 1) & 1;
        if (!pa_wait(&s.p_full[pb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA) ||
            !pa_wait(&s.v_full[pb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA) ||
            !pa_wait(&s.o_empty[pb], ph ^ 1, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint32_t pa = smem_u32(s.p[pb]), va = smem_u32(s.v[pb]);
#pragma unroll
        for (int kk = 0; kk < kPaTile / 16; ++kk) {
          const uint64_t ad = sdesc_k_sw128(pa + (kk >> 2) * PaSmem<D>::kHalf + (kk & 3) * 32);
          const uint64_t bd = sdesc_mn_sw128(va + kk * 16 * 128, PaSmem<D>::kHalf, 1024);
          mma_f16(tmem + 256 + pb * 128, ad, bd, kIdPV, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s.o_full[pb]);
        tc_commit(&s.p_empty[pb]);
        tc_commit(&s.v_empty[pb]);
        return true;
      };
      bool ok = pa_wait(&s.q_full, 0, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA);
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!pa_wait(&s.k_full[st], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA) ||
            !pa_wait(&s.s_empty[st], ph ^ 1, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t ka = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * PaSmem<D>::kHalf + (kk & 3) * 32;
          mma_f16(tmem + st * 128, sdesc_k_sw128(q_addr + off), sdesc_k_sw128(ka + off), kIdQK,
                  kk > 0 ? 1u : 0u);
        }
        tc_commit(&s.s_full[st]);
        tc_commit(&s.k_empty[st]);
        if (j > 0) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(n_tiles - 1);
      tc_commit(&s.mma_done);  // arrives once every MMA issued above has completed
      mbar_wait(&s.mma_done, 0, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
    }
    __syncwarp();
  } else {
    // -------------------------------------------- softmax and correction
    const int r = threadIdx.x;  // query row of the tile = TMEM lane
    const uint32_t lane_tm = tmem + ((uint32_t)(warp * 32) << 16);
    const int q_row = q0 + r;
    const int lim = q_row < q_len ? min(ctx, prefix + q_row + 1) : 0;  // keys [0, lim) visible
    const int swz = r & 7;
    const uint32_t prow = (uint32_t)(r >> 3) * 1024 + (uint32_t)swz * 128;
    float acc[D];
#pragma unroll
    for (int c = 0; c < D; ++c) acc[c] = 0.f;
    float m = -FLT_MAX, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int sb = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!pa_wait(&s.s_full[sb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_tm = lane_tm + sb * 128;
      const int kb = j * kPaTile;
      float mx = -FLT_MAX;
#pragma unroll 1
      for (int c = 0; c < kPaTile / 32; ++c) {
        uint32_t v[32];
        tmem_ld_x32(s_tm + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float x = kb + c * 32 + e < lim ? __fmul_rn(__uint_as_float(v[e]), p.scale) : -FLT_MAX;
          mx = fmaxf(mx, x);
        }
      }
      const float m_new = fmaxf(m, mx);
      if (j >= 2 && !pa_wait(&s.p_empty[sb], ((j >> 1) - 1) & 1, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) {
        ok = false;
        break;
      }
      uint8_t* const pbuf = s.p[sb];
      float lsum = 0.f;
#pragma unroll 1
      for (int c = 0; c < kPaTile / 32; ++c) {
        uint32_t v[32];
        tmem_ld_x32(s_tm + c * 32, v);
        tmem_wait_ld();
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int pos = kb + c * 32 + e;
          const float x0 = pos < lim ? __fmul_rn(__uint_as_float(v[e]), p.scale) : -FLT_MAX;
          const float x1 = pos + 1 < lim ? __fmul_rn(__uint_as_float(v[e + 1]), p.scale) : -FLT_MAX;
          const float p0 = __expf(x0 - m_new), p1 = __expf(x1 - m_new);
          lsum += p0;
          lsum += p1;
          const __half2 hp = __floats2half2_rn(p0, p1);
          packed[e >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
        }
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int c8 = c * 4 + qd;  // 8-key chunk of the row
          *reinterpret_cast<uint4*>(pbuf + (c8 >> 3) * PaSmem<D>::kHalf + prow + (((c8 & 7) ^ swz) << 4)) =
              make_uint4(packed[qd * 4], packed[qd * 4 + 1], packed[qd * 4 + 2], packed[qd * 4 + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s.s_empty[sb]);
      const float alpha = __expf(m - m_new);
      l = fmaf(l, alpha, lsum);
      m = m_new;
      if (j == n_tiles - 1 && kv_end < kb + kPaTile) {
        // keys past the context in the last tile: zero their V rows (pool
        // slots that may hold anything) so that 0-probability keys add 0
        if (!pa_wait(&s.v_full[sb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        if (r >= kv_end - kb) {
#pragma unroll
          for (int hf = 0; hf < D / 64; ++hf) {
            uint4* row = reinterpret_cast<uint4*>(s.v[sb] + hf * PaSmem<D>::kHalf + r * 128);
#pragma unroll
            for (int c = 0; c < 8; ++c) row[c] = make_uint4(0, 0, 0, 0);
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&s.p_full[sb]);
      if (j > 0 && !pa_correct<D>(s, acc, j - 1, alpha_prev, lane_tm + 256, p.status)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok) ok = pa_correct<D>(s, acc, n_tiles - 1, alpha_prev, lane_tm + 256, p.status);
    if (ok && q_row < q_len) {
      uint4* dst = reinterpret_cast<uint4*>(p.out + (size_t)(q_start + q_row) * p.ld_out + (size_t)h * D);
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const __half2 hv = __floats2half2_rn(__fdiv_rn(acc[c * 8 + 2 * e], l), __fdiv_rn(acc[c * 8 + 2 * e + 1], l));
          w[e] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kPaTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 pa_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

// fp16 [rows][heads][D] (token stride ld elements, heads contiguous) as a 3-D
// tensor map with a (64, 1, box_rows) box and the 128-byte swizzle.
int make_rows_map(CUtensorMap* map, const void* base, long long rows, int heads, int D, long long ld,
                  int box_rows, const char* what) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = pa_encode_fn();
  if (!fn) return fail(NPL_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)ld * 2};
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)box_rows};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NPL_ERR_ARG, "cuTensorMapEncodeTiled (%s) failed (%d)", what, (int)r);
  return NPL_OK;
}

int gcd_int(int a, int b) {
  while (b) {
    const int t = a % b;
    a = b;
    b = t;
  }
  return a;
}

template <int D>
int launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const PaArgs& p, int B,
                   int n_qtiles, cudaStream_t st) {
  const int smem = (int)sizeof(PaSmem<D>) + 1024;
  if (cudaFuncSetAttribute(prefill_attn_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status("npl_paged_prefill_attention: smem attribute");
  return launch_pdl("npl_paged_prefill_attention", prefill_attn_kernel<D>, dim3(n_qtiles, B, p.H),
                    dim3(kPaThreads), (size_t)smem, st, tq, tk, tv, p);
}

}  // namespace
}  // namespace npl

using namespace npl;

extern "C" int npl_paged_prefill_attention(const void* q, int ld_q, int total_q, int H, int Hkv, int D,
                                           const void* k_cache, const void* v_cache, int num_blocks,
                                           int block_size, const int32_t* block_tables, int bt_stride,
                                           int max_blocks, const int32_t* context_lens, const int32_t* q_lens,
                                           const int32_t* q_offsets, int B, int max_q_len, float scale, void* out,
                                           int ld_out, void* stream) {
  if (int rc = check_device()) return rc;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !q_lens || !q_offsets || !out)
    return fail(NPL_ERR_ARG, "npl_paged_prefill_attention: null pointer");
  if (total_q < 0 || B < 0 || max_q_len < 0 || H <= 0 || Hkv <= 0 || H % Hkv || num_blocks <= 0 ||
      block_size <= 0 || max_blocks <= 0 || bt_stride < max_blocks || ld_q < H * D || ld_out < H * D ||
      ld_q % 8 || ld_out % 8)
    return fail(NPL_ERR_ARG, "npl_paged_prefill_attention: bad shape");
  if (D != 128 && D != 64)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_prefill_attention: head_dim %d (64 or 128)", D);
  if (block_size % 8)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_prefill_attention: block_size %d (a multiple of 8)", block_size);
  if ((long long)num_blocks * block_size >= (1ll << 31) || (long long)max_blocks * block_size >= (1ll << 31) ||
      (long long)total_q >= (1ll << 31) - kPaTile)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_prefill_attention: pool or batch too large for 32-bit rows");
  for (const void* p : std::initializer_list<const void*>{q, k_cache, v_cache, out})
    if (!aligned16(p)) return fail(NPL_ERR_ARG, "npl_paged_prefill_attention: pointers must be 16-byte aligned");
  if (B == 0 || total_q == 0 || max_q_len == 0) return NPL_OK;
  const int n_qtiles = (max_q_len + kPaTile - 1) / kPaTile;
  if (n_qtiles > kPaMaxQTiles || B > 65535 || H > 65535)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_prefill_attention: launch shape too large");
  const int piece = gcd_int(block_size, kPaTile);
  CUtensorMap tq, tk, tv;
  if (int rc = make_rows_map(&tq, q, total_q, H, D, ld_q, kPaTile, "q")) return rc;
  if (int rc = make_rows_map(&tk, k_cache, (long long)num_blocks * block_size, Hkv, D, (long long)Hkv * D, piece,
                             "K cache"))
    return rc;
  if (int rc = make_rows_map(&tv, v_cache, (long long)num_blocks * block_size, Hkv, D, (long long)Hkv * D, piece,
                             "V cache"))
    return rc;
  PaArgs p{};
  p.out = static_cast<__half*>(out);
  p.ld_out = ld_out;
  p.bt = block_tables;
  p.bt_stride = bt_stride;
  p.max_blocks = max_blocks;
  p.ctx_lens = context_lens;
  p.q_lens = q_lens;
  p.q_offsets = q_offsets;
  p.H = H;
  p.Hkv = Hkv;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.piece = piece;
  p.total_q = total_q;
  p.scale = scale;
  p.status = device_status_ptr();
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return D == 128 ? launch_prefill<128>(tq, tk, tv, p, B, n_qtiles, st)
                  : launch_prefill<64>(tq, tk, tv, p, B, n_qtiles, st);
}
