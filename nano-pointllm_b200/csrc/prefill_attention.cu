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
// Scores are fp32 dot products of the fp16 rows times `scale` (> 0), masked
// to the lowest float; the softmax runs online over key tiles:
//   m' = max(m, rowmax(s));  p = exp(s - m');  alpha = exp(m - m')
//   acc = acc * alpha + fp16(p) . V  (fp32 accumulation);  l = l * alpha + sum(p)
// and out = fp16(acc / l). The probabilities are rounded to fp16 for the
// P.V product and summed unrounded into l, as the reference does. Its key
// tile is 64 (here 128), exp(x) is evaluated here as exp2(x * log2(e)) with
// the scale folded into one FMA, acc / l as acc * (1 / l), and the fp32 sums
// run in another order: results agree to fp16 rounding, not bit for bit.
//
// Persistent: one CTA per SM walks the (128-query tile, sequence, head)
// items with a stride of the grid, longest first; the K/V rings, TMEM buffers
// and barrier phases run on across items, so the next item's loads and
// first Q.K^T overlap the current item's last tiles. 320 threads:
//   warp 8      TMA: the Q tile once, then 128-key K and V tiles through the
//               block table (2-stage rings; pieces of gcd(block_size, 128)
//               keys, 128-byte swizzle); keys past the tile's last visible
//               key are zero-filled out-of-bounds loads;
//   warp 9      MMA issue (one thread): S_j = Q K_j^T into one of two TMEM
//               buffers, then O_{j-1} = P_{j-1} V_{j-1} (V is the MN-major B
//               operand: the cache layout as is) into one of two TMEM
//               buffers, so the tensor core works on tile j while the
//               softmax warps work on tile j-1;
//   warps 0-7   two warpgroups per query row (TMEM lane = row): group g
//               takes keys [64g, 64g + 64) of each tile -- partial row max,
//               combined with the other group's through shared memory, then
//               exp and its half of fp16 P_j (K-major, 128-byte swizzle: the
//               A operand of P.V) -- and the head-dimension half g of the
//               output: acc = acc * alpha + O_{j-1} in registers, finally
//               out = acc * (1 / l) (l summed per group, combined at the end).
// TMEM: S at columns [0, 256), O at [256, 512).
#include <algorithm>
#include <cfloat>
#include <initializer_list>

#include <cudaTypedefs.h>

#include "npl_common.cuh"

namespace npl {
namespace {

constexpr int kPaTile = 128;
constexpr int kPaThreads = 320;  // warps 0-7 softmax, 8 TMA, 9 MMA
constexpr uint32_t kPaTmemCols = 512;

template <int D>
struct PaSmem {
  static constexpr uint32_t kHalf = kPaTile * 128;        // 128 rows x 64 fp16 (one swizzle span)
  static constexpr uint32_t kTileBytes = kPaTile * D * 2;  // Q / K / V tile
  static constexpr uint32_t kPBytes = kPaTile * kPaTile * 2;
  alignas(1024) uint8_t q[kTileBytes];
  alignas(1024) uint8_t k[2][kTileBytes];
  alignas(1024) uint8_t v[2][kTileBytes];
  alignas(1024) uint8_t p[kPBytes];  // P of one key tile (the A operand of P.V)
  uint64_t q_full, q_empty;
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2], p_full, p_empty, o_full[2], o_empty[2];
  uint64_t mma_done;
  uint64_t red_bar[2];           // the two softmax groups' partial maxima of a tile are in
  uint64_t red_done;             // both partial normalisers are in
  float red_max[2][2][kPaTile];  // [tile parity][key half][row]: partial row maxima
  float red_l[2][kPaTile];       // [key half][row]: partial normalisers at the end
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

// 2^x (ex2.approx.ftz: results below 2^-126 flush to 0; every p and alpha
// here is such a value or one fp16 keeps, and a flushed term adds < 2^-126).
__device__ __forceinline__ float pa_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

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

// acc = acc * alpha + O_i over this thread's half of the head dimension
// (TMEM buffer i & 1, this thread's lane, columns [col0, col0 + D/2)).
template <int D>
__device__ __forceinline__ bool pa_correct(PaSmem<D>& s, float (&acc)[D / 2], int i, float alpha, uint32_t o_tm,
                                           int* status) {
  const int ob = i & 1;
  if (!pa_wait(&s.o_full[ob], (i >> 1) & 1, &s.abort, status, NPL_DEV_TIMEOUT_EPILOGUE)) return false;
  tc_fence_after();
  uint32_t v[D / 2];
#pragma unroll
  for (int c = 0; c < D / 64; ++c) tmem_ld_x32(o_tm + ob * 128 + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
  tmem_wait_ld();
#pragma unroll
  for (int e = 0; e < D / 2; ++e) acc[e] = fmaf(acc[e], alpha, __uint_as_float(v[e]));
  tc_fence_before();
  mbar_arrive(&s.o_empty[ob]);
  return true;
}

// One work item: 128 query rows of one (sequence, head). Every role of the
// CTA decodes the same items from the same read-only metadata, so all agree
// on which items have work and how many key tiles each has.
struct PaItem {
  int b, h, q0, q_len, ctx, q_start, prefix, rows, kv_end, n_tiles;
  bool skip;  // no query row of this item exists (or its offsets are invalid)
};

// Item i of the launch, longest first: items [0, B*H) are the last query
// tiles of every (sequence, head), the next B*H the tiles before, and so on.
__device__ __forceinline__ PaItem pa_item(const PaArgs& p, int i, int n_qtiles, int B) {
  PaItem it;
  const int bh = B * p.H;
  const int level = i / bh, rem = i - level * bh;
  it.b = rem / p.H;
  it.h = rem - it.b * p.H;
  it.q0 = (n_qtiles - 1 - level) * kPaTile;
  it.q_len = p.q_lens[it.b];
  it.skip = it.q0 >= it.q_len;
  it.ctx = p.ctx_lens[it.b];
  it.q_start = p.q_offsets[it.b];
  it.prefix = it.ctx - it.q_len;
  it.rows = min(kPaTile, it.q_len - it.q0);
  it.kv_end = min(it.ctx, it.prefix + it.q0 + it.rows);  // keys some row of the item sees
  it.n_tiles = it.kv_end > 0 ? (it.kv_end + kPaTile - 1) / kPaTile : 0;
  if (!it.skip && (it.q_start < 0 || it.q_start > p.total_q - it.q_len)) it.skip = true;  // rows outside q / out
  if (it.skip) it.n_tiles = 0;
  return it;
}

template <int D>
__global__ void __launch_bounds__(kPaThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const PaArgs p, int n_items, int n_qtiles,
                        int B) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  PaSmem<D>& s = *reinterpret_cast<PaSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    mbar_init(&s.q_empty, 1);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_empty[i], 256);
      mbar_init(&s.o_full[i], 1);
      mbar_init(&s.o_empty[i], 256);
    }
    mbar_init(&s.p_full, 256);
    mbar_init(&s.p_empty, 1);
    mbar_init(&s.mma_done, 1);
    mbar_init(&s.red_bar[0], 256);
    mbar_init(&s.red_bar[1], 256);
    mbar_init(&s.red_done, 256);
    s.abort = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&s.tmem_base, kPaTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  pdl_wait();  // q, the pool and the metadata come from earlier work on the stream
  pdl_trigger();

  if (warp == 8) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      prefetch_tensormap(&tmap_q);
      prefetch_tensormap(&tmap_k);
      prefetch_tensormap(&tmap_v);
      const uint64_t pol_q = policy_evict_first();
      const uint64_t pol_kv = policy_evict_normal();  // re-read by the other query tiles of the sequence
      const int oob = p.num_blocks * p.block_size;
      int kt = 0, nk = 0, nv = 0, nq = 0;  // tiles of this CTA so far; K, V tiles and Q tiles issued
      bool ok = true;
      for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
        const PaItem it = pa_item(p, i, n_qtiles, B);
        if (it.n_tiles == 0) continue;
        if (it.prefix < 0 || it.ctx > p.max_blocks * p.block_size) atomicCAS(p.status, 0, NPL_DEV_BAD_INDEX);
        const int kvh = it.h / (p.H / p.Hkv);
        const int32_t* table = p.bt + (size_t)it.b * p.bt_stride;
        if (nq > 0 && !pa_wait(&s.q_empty, (nq - 1) & 1, &s.abort, p.status, NPL_DEV_TIMEOUT_TMA)) break;
        mbar_arrive_expect_tx(&s.q_full, PaSmem<D>::kTileBytes);
#pragma unroll
        for (int hf = 0; hf < D / 64; ++hf)
          tma_load_3d(s.q + hf * PaSmem<D>::kHalf, &tmap_q, hf * 64, it.h, it.q_start + it.q0, &s.q_full, pol_q);
        ++nq;
        for (int j = 0; j < it.n_tiles; ++j, ++kt) {
          const int st = kt & 1;
          const uint32_t ph = (kt >> 1) & 1;
          if (!pa_wait(&s.k_empty[st], ph ^ 1, &s.abort, p.status, NPL_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.k_full[st], PaSmem<D>::kTileBytes);
          load_kv_tile<D>(s.k[st], &tmap_k, p, table, j, it.kv_end, kvh, oob, &s.k_full[st], pol_kv);
          nk = kt + 1;
          if (!pa_wait(&s.v_empty[st], ph ^ 1, &s.abort, p.status, NPL_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.v_full[st], PaSmem<D>::kTileBytes);
          load_kv_tile<D>(s.v[st], &tmap_v, p, table, j, it.kv_end, kvh, oob, &s.v_full[st], pol_kv);
          nv = kt + 1;
        }
      }
      // Drain: every load issued here has landed before the CTA may exit
      // (already true unless a role gave up). The last load of each stage is
      // the newest phase of its barrier.
      if (nq > 0) mbar_wait(&s.q_full, (nq - 1) & 1, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
      for (int j = max(0, nk - 2); j < nk; ++j)
        mbar_wait(&s.k_full[j & 1], (j >> 1) & 1, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
      for (int j = max(0, nv - 2); j < nv; ++j)
        mbar_wait(&s.v_full[j & 1], (j >> 1) & 1, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_f16(kPaTile, kPaTile, false);
      constexpr uint32_t kIdPV = idesc_f16(kPaTile, D, true);
      const uint32_t q_addr = smem_u32(s.q);
      // O_t = P_t V_t for the global tile index t of this CTA
      auto issue_pv = [&](int t) -> bool {
        const int pb = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!pa_wait(&s.p_full, t & 1, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA) ||
            !pa_wait(&s.v_full[pb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA) ||
            !pa_wait(&s.o_empty[pb], ph ^ 1, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA))
          return false;
        tc_fence_after();
        const uint32_t pa = smem_u32(s.p), va = smem_u32(s.v[pb]);
#pragma unroll
        for (int kk = 0; kk < kPaTile / 16; ++kk) {
          const uint64_t ad = sdesc_k_sw128(pa + (kk >> 2) * PaSmem<D>::kHalf + (kk & 3) * 32);
          const uint64_t bd = sdesc_mn_sw128(va + kk * 16 * 128, PaSmem<D>::kHalf, 1024);
          mma_f16(tmem + 256 + pb * 128, ad, bd, kIdPV, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s.o_full[pb]);
        tc_commit(&s.p_empty);
        tc_commit(&s.v_empty[pb]);
        return true;
      };
      bool ok = true;
      int kt = 0, nq = 0, pending = -1;  // pending: tile whose P.V is issued after the next Q.K^T
      for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
        const PaItem it = pa_item(p, i, n_qtiles, B);
        if (it.n_tiles == 0) continue;
        if (!pa_wait(&s.q_full, nq & 1, &s.abort, p.status, NPL_DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        ++nq;
        for (int j = 0; j < it.n_tiles; ++j, ++kt) {
          const int st = kt & 1;
          const uint32_t ph = (kt >> 1) & 1;
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
          if (j == it.n_tiles - 1) tc_commit(&s.q_empty);  // the item's Q is no longer read
          if (pending >= 0 && !issue_pv(pending)) {
            ok = false;
            break;
          }
          pending = kt;
        }
      }
      if (ok && pending >= 0) issue_pv(pending);
      tc_commit(&s.mma_done);  // arrives once every MMA issued above has completed
      mbar_wait(&s.mma_done, 0, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
    }
    __syncwarp();
  } else {
    // -------------------------------------------- softmax and correction
    // Two warpgroups share every query row: group g owns keys [64g, 64g + 64)
    // of each key tile (its half of P) and the head-dimension half
    // [g D/2, (g+1) D/2) of the output; the row max is combined per tile
    // through shared memory, the normaliser once per item.
    const int g = warp >> 2;
    const int r = threadIdx.x & 127;  // query row of the item = TMEM lane
    const uint32_t lane_tm = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t o_tm = lane_tm + 256 + g * (D / 2);
    const int swz = r & 7;
    const uint32_t prow = (uint32_t)(r >> 3) * 1024 + (uint32_t)swz * 128;
    const float c2 = p.scale * 1.4426950408889634f;  // scale * log2(e)
    bool ok = true;
    int kt = 0, nitems = 0;
    for (int i = blockIdx.x; ok && i < n_items; i += gridDim.x) {
      const PaItem it = pa_item(p, i, n_qtiles, B);
      if (it.skip) {
        if (it.q0 < it.q_len && threadIdx.x == 0) atomicCAS(p.status, 0, NPL_DEV_BAD_INDEX);
        continue;
      }
      const int q_row = it.q0 + r;
      __half* const dst_row = p.out + (size_t)(it.q_start + q_row) * p.ld_out + (size_t)it.h * D + g * (D / 2);
      if (it.n_tiles == 0) {  // no visible key: the reference's masked loads make the output 0
        if (q_row < it.q_len) {
#pragma unroll
          for (int c = 0; c < D / 16; ++c) reinterpret_cast<uint4*>(dst_row)[c] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const int lim = q_row < it.q_len ? min(it.ctx, it.prefix + q_row + 1) : 0;  // keys [0, lim) visible
      float acc[D / 2];
#pragma unroll
      for (int c = 0; c < D / 2; ++c) acc[c] = 0.f;
      float m = -FLT_MAX, l = 0.f, alpha_prev = 0.f;  // m: running max of the raw scores
      for (int j = 0; j < it.n_tiles; ++j) {
        const int t = kt + j;  // this CTA's tile index: ring, buffer and phase selector
        const int sb = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!pa_wait(&s.s_full[sb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int kb = j * kPaTile + g * 64;  // first key of this thread's half tile
        uint32_t v[64];
        tmem_ld_x32(lane_tm + sb * 128 + g * 64, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld_x32(lane_tm + sb * 128 + g * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_wait_ld();
        // Scores stay raw: max(s * scale) = max(s) * scale for scale > 0, and
        // exp(s * scale - m') = exp2(fma(s, c2, -m_raw' * c2)), c2 = scale * log2(e).
        if (kb + 64 > lim) {
#pragma unroll
          for (int e = 0; e < 64; ++e)
            if (kb + e >= lim) v[e] = __float_as_uint(-FLT_MAX);
        }
        float mxp[8];  // independent partial maxima (short dependency chains)
#pragma unroll
        for (int e = 0; e < 8; ++e) mxp[e] = __uint_as_float(v[e]);
#pragma unroll
        for (int e = 8; e < 64; ++e) mxp[e & 7] = fmaxf(mxp[e & 7], __uint_as_float(v[e]));
        s.red_max[sb][g][r] = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                    fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
        mbar_arrive(&s.red_bar[sb]);  // release: the partial max above is visible to the waiters
        if (!pa_wait(&s.red_bar[sb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        const float m_new = fmaxf(m, fmaxf(s.red_max[sb][0][r], s.red_max[sb][1][r]));
        const float neg_mc = -m_new * c2;
        if (t >= 1 && !pa_wait(&s.p_empty, (t - 1) & 1, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        float lsp[8];  // independent partial sums
#pragma unroll
        for (int e = 0; e < 8; ++e) lsp[e] = 0.f;
        uint32_t packed[32];
#pragma unroll
        for (int e = 0; e < 64; e += 2) {
          const float p0 = pa_exp2(fmaf(__uint_as_float(v[e]), c2, neg_mc));
          const float p1 = pa_exp2(fmaf(__uint_as_float(v[e + 1]), c2, neg_mc));
          lsp[(e >> 1) & 7] += p0;
          lsp[((e >> 1) + 4) & 7] += p1;
          const __half2 hp = __floats2half2_rn(p0, p1);
          packed[e >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
        }
        uint8_t* const pbuf = s.p + g * PaSmem<D>::kHalf;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8)  // 8-key chunks of the row's half
          *reinterpret_cast<uint4*>(pbuf + prow + ((c8 ^ swz) << 4)) =
              make_uint4(packed[c8 * 4], packed[c8 * 4 + 1], packed[c8 * 4 + 2], packed[c8 * 4 + 3]);
        tc_fence_before();
        mbar_arrive(&s.s_empty[sb]);
        const float lsum = ((lsp[0] + lsp[1]) + (lsp[2] + lsp[3])) + ((lsp[4] + lsp[5]) + (lsp[6] + lsp[7]));
        const float alpha = pa_exp2(fmaf(m, c2, neg_mc));
        l = fmaf(l, alpha, lsum);
        m = m_new;
        const int tile0 = j * kPaTile;
        if (j == it.n_tiles - 1 && it.kv_end < tile0 + kPaTile && g < D / 64) {
          // keys past the context in the last tile: zero their V rows (pool
          // slots that may hold anything) so that 0-probability keys add 0
          if (!pa_wait(&s.v_full[sb], ph, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) {
            ok = false;
            break;
          }
          if (r >= it.kv_end - tile0) {
            uint4* row = reinterpret_cast<uint4*>(s.v[sb] + g * PaSmem<D>::kHalf + r * 128);
#pragma unroll
            for (int c = 0; c < 8; ++c) row[c] = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&s.p_full);
        if (j > 0 && !pa_correct<D>(s, acc, t - 1, alpha_prev, o_tm, p.status)) {
          ok = false;
          break;
        }
        alpha_prev = alpha;
      }
      if (ok) ok = pa_correct<D>(s, acc, kt + it.n_tiles - 1, alpha_prev, o_tm, p.status);
      s.red_l[g][r] = l;
      mbar_arrive(&s.red_done);  // every softmax thread arrives once per item, whatever happened above
      if (ok) ok = pa_wait(&s.red_done, nitems & 1, &s.abort, p.status, NPL_DEV_TIMEOUT_EPILOGUE);
      const float inv_l = __frcp_rn(s.red_l[0][r] + s.red_l[1][r]);  // out = acc * (1 / l)
      if (ok && q_row < it.q_len) {
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __half2 hv = __floats2half2_rn(__fmul_rn(acc[c * 8 + 2 * e], inv_l),
                                                 __fmul_rn(acc[c * 8 + 2 * e + 1], inv_l));
            w[e] = *reinterpret_cast<const uint32_t*>(&hv);
          }
          reinterpret_cast<uint4*>(dst_row)[c] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      kt += it.n_tiles;
      ++nitems;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
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
  const long long items = (long long)n_qtiles * B * p.H;
  const int sms = num_sms();
  const int grid = (int)std::min<long long>(items, sms > 0 ? sms : 148);  // persistent: one CTA per SM
  return launch_pdl("npl_paged_prefill_attention", prefill_attn_kernel<D>, dim3(grid), dim3(kPaThreads),
                    (size_t)smem, st, tq, tk, tv, p, (int)items, n_qtiles, B);
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
  if (!(scale > 0.f) || !(scale < 3.0e38f))
    return fail(NPL_ERR_ARG, "npl_paged_prefill_attention: scale must be positive and finite");
  if (block_size % 8)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_prefill_attention: block_size %d (a multiple of 8)", block_size);
  if ((long long)num_blocks * block_size >= (1ll << 31) || (long long)max_blocks * block_size >= (1ll << 31) ||
      (long long)total_q >= (1ll << 31) - kPaTile)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_prefill_attention: pool or batch too large for 32-bit rows");
  for (const void* p : std::initializer_list<const void*>{q, k_cache, v_cache, out})
    if (!aligned16(p)) return fail(NPL_ERR_ARG, "npl_paged_prefill_attention: pointers must be 16-byte aligned");
  if (B == 0 || total_q == 0 || max_q_len == 0) return NPL_OK;
  const int n_qtiles = (max_q_len + kPaTile - 1) / kPaTile;
  if ((long long)n_qtiles * B * H >= (1ll << 31))
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_prefill_attention: too many (query tile, sequence, head) items");
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
