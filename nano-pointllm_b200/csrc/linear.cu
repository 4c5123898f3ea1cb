// W8A8 linear on the 5th-generation tensor cores (tcgen05, kind::i8).
//
// Replaces w8a8.py:118-139 (integer_linear_per_output_reference) and the
// F.linear projection call sites of the decode/prefill path (packed QKV, O,
// packed gate/up + act_fn(gate) * up, down, LM head), with the layer math
// around them fused in:
//   activations: int8 via TMA, or quantised in the kernel from fp16 rows,
//                optionally RMSNorm-ed first (lightweight_runner.py:239-245)
//   epilogues:   dequant; + residual; SiLU(gate) * up (+ per-token absmax of
//                the result); RoPE + KV-cache store (paged_attention.py:
//                1284-1294)
//
// Formulation ("swap AB"): the weight tile is the MMA's A operand and the
// tokens are its N dimension,
//     D[n, m] = sum_k W[n, k] * X[m, k]      (A = W: 128 rows, B = X: NT rows)
// so a decode batch of M <= 64 tokens fills an MMA of 128 x NT x 32 with
// NT = 8..64, and prefill uses NT = 128/256 token tiles.
//
// Per CTA (192 threads, one CTA per SM):
//   warp 0     TMA producer: weight tile [128 rows x 128 B] (+ token tile
//              [NT x 128 B] for int8 activations) per stage, 128-byte swizzle,
//              a ring of 3-12 stages in shared memory
//   warp 1     TMEM owner + MMA issuer (one thread): 4 MMAs of K = 32 per
//              stage into a ring of 2-4 int32 accumulators in TMEM
//   warps 2-5  before the main loop: quantise fp16 activations (with RMSNorm)
//              into per-unit token tiles in shared memory; then the epilogue:
//              tcgen05.ld (TMEM lane = weight row, column = token), dequant
//              ((acc * sa) * sw + bias) and the fused tail
//
// Work split, decode tiles (NT <= 64): cluster split-K. Each tile's k-blocks
// are shared by the S CTAs of one thread-block cluster (S <= 8, chosen per
// shape); clusters take tiles round-robin. The non-leader CTAs add their
// int32 partial tiles into the leader's shared memory with one bulk DSMEM
// reduction each, so the cross-CTA reduction never leaves the GPC.
//
// Work split, prefill tiles (NT >= 128), and the fallback when the clusters
// do not fit at once: stream-K. The (tile, k-block) units of the whole
// problem are divided evenly over the grid. A CTA that owns a whole tile runs
// its epilogue from TMEM; partial tiles are reduced through int32 atomics in
// the caller's workspace (exact and order-independent), and the CTA whose
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
#include <atomic>
#include <initializer_list>
#include <mutex>
#include <vector>

#include "npl_common.cuh"

namespace npl {
namespace {

constexpr int kTileN = 128;   // weight rows per tile (MMA M)
constexpr int kBlockK = 128;  // K bytes per stage (one 128-byte swizzle atom)
// Epilogue warpgroups: prefill tiles (NT >= 128) take two, each draining half
// of the tile's token columns (the epilogue of a 256-token tile is longer than
// its main loop with one); decode tiles take one.
__host__ __device__ constexpr int epi_groups_for(int nt) { return nt >= 128 ? 2 : 1; }
__host__ __device__ constexpr int threads_for(int nt) { return 64 + 128 * epi_groups_for(nt); }
constexpr int kMaxStages = 12;
constexpr int kMaxAccBufs = 4;
constexpr int kCoresidentSmem = 110 * 1024;  // two CTAs per SM (programmatic dependent launch)
constexpr int kMaxSmem = 226 * 1024;

struct LinearArgs {
  int M, N, K;
  int x_mode;
  const float* sa;         // NPL_X_INT8: per-token scales
  const __half* xf;        // NPL_X_F16_*: fp16 activations [M, K]
  int ldx;
  int32_t* x_absmax;       // NPL_X_F16_ABSMAX: per-token absmax (float bits); zeroed after use
  const __half* norm_w;    // NPL_X_F16_RMSNORM
  float eps;
  const float* sw;
  const float* bias;
  int epilogue;
  const __half* residual;
  int ld_res;
  void* out;
  int ld_out;
  int out_dtype;
  int32_t* acc_out;
  int32_t* absmax_out;     // NPL_EPI_SILU_MUL: per-token max |out| (float bits), atomic max
  int8_t* silu_q;          // NPL_EPI_SILU_MUL with absmax_out: per-token int8 of out [M, N/2] (row stride N/2)
  float* silu_qs;          //   and its scales [M], written after every CTA has stored its outputs
  const __half* cos_t;     // NPL_EPI_ROPE_KV
  const __half* sin_t;
  int max_position;
  const int64_t* positions;
  const int32_t* slots;
  __half* q_out;
  __half* k_cache;
  __half* v_cache;
  long long num_slots;
  int heads, kv_heads, head_dim;
  int n_tiles;
  int k_blocks;
  long long total_units;
  int split;      // > 0: cluster split-K with `split` CTAs per cluster; 0: stream-K
  int clusters;   // cluster split-K: number of clusters (tile stride)
  int tiles;      // m_tiles * n_tiles
  int red_bufs;   // cluster split-K: partial-tile buffers (1 or 2)
  int dp_tiles;   // stream-K: tiles [0, dp_tiles) run whole, CTA b taking b, b + grid, ...
  int raster_g;   // token tiles per raster group (tile numbering, see tile_coords)
  long long sk_units;  // stream-K units after the whole tiles: (tiles - dp_tiles) * k_blocks
  int stages;
  int x_slots;
  uint32_t off_a, off_b, off_x, off_f, off_r;
  int32_t* ws_acc;   // [grid - 1 slots][NT][128]
  int32_t* ws_cnt;   // [grid - 1 slots]
  int32_t* ws_xcnt;  // [1]: CTAs done reading x_absmax
  int32_t* ws_gcnt;  // [2]: CTAs arrived at / done after the grid-wide step of silu_q
  int* status;
};

// Control block at the start of the dynamic shared memory; the stage ring,
// the token tiles and the scale scratch follow at the offsets in LinearArgs.
struct LinearCtl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tfull[kMaxAccBufs];
  uint64_t tempty[kMaxAccBufs];
  uint64_t teardown;
  uint64_t xready;
  uint64_t rfull[2];  // cluster leader: contributors' partials of buffer b landed
  uint64_t rfree[2];  // cluster contributor: leader consumed buffer b
  uint32_t tmem_base;
  int last_flag;
  __half xchg[2][8][kTileN];  // epilogue exchange between TMEM lanes, per warpgroup
};

// TMEM accumulator ring depth: decode tiles keep 4 accumulators so that the
// MMAs run up to 3 tiles ahead of an epilogue that waits for its cluster;
// prefill tiles (NT >= 128) keep 2 (the 512 TMEM columns bound 2 x 256).
__host__ __device__ constexpr int acc_bufs_for(int nt) { return nt <= 64 ? 4 : 2; }

__host__ __device__ constexpr uint32_t tmem_cols_for(int nt) {
  uint32_t c = 32;
  while (c < (uint32_t)(acc_bufs_for(nt) * nt)) c <<= 1;
  return c;
}

// Epilogue warpgroup of this thread (warps 2-5: 0, warps 6-9: 1) and its
// named barrier; epi_all_bar() joins every epilogue warp of the CTA.
template <int NT>
__device__ __forceinline__ int epi_group() {
  if constexpr (epi_groups_for(NT) == 1) return 0;
  return (int)(threadIdx.x - 64) >> 7;
}
template <int NT>
__device__ __forceinline__ void epi_bar() {
  if constexpr (epi_groups_for(NT) == 1)
    asm volatile("bar.sync 1, 128;" ::: "memory");
  else
    asm volatile("bar.sync %0, 128;" ::"r"(1 + epi_group<NT>()) : "memory");
}
__device__ __forceinline__ void epi_all_bar(int groups) {
  asm volatile("bar.sync 3, %0;" ::"r"(128 * groups) : "memory");
}

// Tile t of the numbering -> (token tile m, weight tile n). Tiles go in groups
// of raster_g token tiles: inside a group the token tile runs fastest, so the
// CTAs working on consecutive tiles at one time share raster_g token tiles and
// about grid / raster_g weight tiles, which L2 then serves to all of them.
// raster_g = 1 is the plain order (weight tile fastest).
template <int NT>
__device__ __forceinline__ void tile_coords(const LinearArgs& p, int t, int& m, int& n) {
  if constexpr (NT <= 64) {  // decode tiles: one raster group (weight tile fastest)
    m = t / p.n_tiles;
    n = t - m * p.n_tiles;
    return;
  }
  const int g = p.raster_g;
  const int span = g * p.n_tiles;
  const int grp = t / span, r = t - grp * span;
  const int m0 = grp * g;
  const int gs = min(g, p.tiles / p.n_tiles - m0);
  m = m0 + r % gs;
  n = r / gs;
}

__device__ __forceinline__ int atomic_add_acq_rel(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Rank of this CTA in its cluster and the k-block range [lo, hi) it owns in
// every tile of the cluster split-K schedule (clusters are consecutive CTAs
// along x).
struct SplitRange {
  int rank, lo, hi;
  __device__ explicit SplitRange(const LinearArgs& p) {
    const int s = max(p.split, 1);
    rank = (int)(blockIdx.x % (unsigned)s);
    lo = rank * p.k_blocks / s;
    hi = (rank + 1) * p.k_blocks / s;
  }
};

// Iterates the CTA's segments (tile, kb0, kb1).
//   stream-K (split == 0): first the whole tiles blockIdx.x, + grid, ... below
//     dp_tiles, then the CTA's contiguous share of the remaining (tile,
//     k-block) units, cut at tile boundaries;
//   cluster split-K: tiles cluster, cluster + clusters, ... with the k-block
//     range of the CTA's rank.
template <int NT>
struct SegmentIter {
  static constexpr bool kWholeTiles = NT >= 128;  // decode tiles run no data-parallel phase
  long long u, u1;
  int k_blocks;
  int tile_next, tile_step, tiles, lo, hi;
  int dp_next, dp_tiles;
  bool split;
  __device__ explicit SegmentIter(const LinearArgs& p) {
    k_blocks = p.k_blocks;
    split = p.split > 0;
    if (split) {
      const SplitRange r(p);
      tile_next = (int)(blockIdx.x / (unsigned)p.split);
      tile_step = p.clusters;
      tiles = p.tiles;
      lo = r.lo;
      hi = r.hi;
      u = u1 = 0;
      dp_next = dp_tiles = 0;
    } else {
      const long long base = (long long)p.dp_tiles * k_blocks;
      u = base + (long long)blockIdx.x * p.sk_units / gridDim.x;
      u1 = base + (long long)(blockIdx.x + 1) * p.sk_units / gridDim.x;
      tile_next = tile_step = tiles = lo = hi = 0;
      dp_next = (int)blockIdx.x;
      dp_tiles = p.dp_tiles;
    }
  }
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (split) {
      if (tile_next >= tiles) return false;
      tile = tile_next;
      tile_next += tile_step;
      kb0 = lo;
      kb1 = hi;
      return true;
    }
    if (kWholeTiles && dp_next < dp_tiles) {
      tile = dp_next;
      dp_next += (int)gridDim.x;
      kb0 = 0;
      kb1 = k_blocks;
      return true;
    }
    if (u >= u1) return false;
    tile = (int)(u / k_blocks);
    kb0 = (int)(u % k_blocks);
    kb1 = (int)min((long long)k_blocks, kb0 + (u1 - u));
    u += kb1 - kb0;
    return true;
  }
};

// ((acc * sa) * sw) + bias_v, the bias added only when the layer has one.
__device__ __forceinline__ float dequant(int32_t acc, float sa, float sw, const float* bias, float bias_v) {
  float v = __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw);
  if (bias) v = __fadd_rn(v, bias_v);
  return v;
}

// Per-row epilogue operands, loaded before the accumulator is ready: the
// weight scale and bias of the row, and the residual of the first 8 tokens.
struct EpiOperands {
  float sw, bias;
  int c_first;  // first token column of the residuals below
  __half res[8];
};

template <int NT>
__device__ __forceinline__ void load_epi_operands(const LinearArgs& p, int m_tile, int n_tile, int row, int c_first,
                                                  EpiOperands& e) {
  const int n = n_tile * kTileN + row;
  e.sw = n < p.N ? p.sw[n] : 0.f;
  e.bias = (p.bias && n < p.N) ? p.bias[n] : 0.f;
  e.c_first = c_first;
  if (p.epilogue == NPL_EPI_RESIDUAL) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = m_tile * NT + c_first + j;
      e.res[j] = (m < p.M && n < p.N) ? p.residual[(size_t)m * p.ld_res + n] : __float2half_rn(0.f);
    }
  }
}

__device__ __forceinline__ void atomic_max_nonneg(int32_t* p, float v) {
  atomicMax(p, __float_as_int(v));  // bit patterns of non-negative floats order like the values
}

// Epilogue of 8 consecutive token columns [c0, c0 + 8) of tile row `row`.
// `sa` holds the per-token activation scales indexed by token.
template <int NT>
__device__ __forceinline__ void epilogue_chunk(const LinearArgs& p, LinearCtl& c, const float* sa, int m_tile,
                                               int n_tile, int row, int c0, const int32_t (&acc)[8],
                                               const EpiOperands& e) {
  const int n = n_tile * kTileN + row;
  const int m_base = m_tile * NT + c0;
  const int lane = threadIdx.x & 31;
  const int eg = epi_group<NT>();
  if (p.acc_out && n < p.N) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (m_base + j < p.M) p.acc_out[(size_t)(m_base + j) * p.N + n] = acc[j];
  }
  if (p.epilogue == NPL_EPI_ROPE_KV) {
    // every tile lies in one of q | k | v (head blocks are multiples of 128)
    const int D = p.head_dim, half_d = D / 2;
    const float sw = e.sw;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = min(m_base + j, p.M - 1);
      c.xchg[eg][j][row] = __float2half_rn(dequant(acc[j], sa[m], sw, p.bias, e.bias));
    }
    epi_bar<NT>();
    const int q_cols = p.heads * D, k_cols = p.kv_heads * D;
    const int d = n % D;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int m = m_base + j;
      if (m >= p.M) break;
      const __half x = c.xchg[eg][j][row];
      const long long slot = p.slots[m];
      const bool slot_ok = slot >= 0 && slot < p.num_slots;
      if (n >= q_cols + k_cols) {  // v
        if (slot_ok) p.v_cache[(slot * p.kv_heads + (n - q_cols - k_cols) / D) * D + d] = x;
        continue;
      }
      const long long pos = p.positions[m];
      if (pos < 0 || pos >= p.max_position) continue;
      const float x1 = __half2float(x);
      const float x2 = __half2float(c.xchg[eg][j][row ^ half_d]);
      const float cs = __half2float(p.cos_t[pos * D + d]);
      const float sn = __half2float(p.sin_t[pos * D + d]);
      // rotate_half(x)[d] = -x[d + D/2] (d < D/2), x[d - D/2] (d >= D/2)
      const float a = __half2float(__float2half_rn(__fmul_rn(x1, cs)));
      const float b = __half2float(__float2half_rn(__fmul_rn(d < half_d ? -x2 : x2, sn)));
      const __half o = __float2half_rn(__fadd_rn(a, b));
      if (n < q_cols)
        p.q_out[((size_t)m * p.heads + n / D) * D + d] = o;
      else if (slot_ok)
        p.k_cache[(slot * p.kv_heads + (n - q_cols) / D) * D + d] = o;
    }
    epi_bar<NT>();
    return;
  }
  if (n >= p.N) return;
  const float sw = e.sw;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int m = m_base + j;
    if (m >= p.M) break;
    const float v = dequant(acc[j], sa[m], sw, p.bias, e.bias);
    if (p.epilogue == NPL_EPI_RESIDUAL) {
      const float o = __half2float(__float2half_rn(v));
      const float r = __half2float(c0 == e.c_first ? e.res[j] : p.residual[(size_t)m * p.ld_res + n]);
      static_cast<__half*>(p.out)[(size_t)m * p.ld_out + n] = __float2half_rn(__fadd_rn(o, r));
    } else if (p.out_dtype == NPL_F32) {
      static_cast<float*>(p.out)[(size_t)m * p.ld_out + n] = v;
    } else {
      static_cast<__half*>(p.out)[(size_t)m * p.ld_out + n] = __float2half_rn(v);
    }
  }
}

// SiLU * up epilogue of token columns [cb, ce) of a tile. Packed gate/up
// layout (w8a8.pack_gate_up): per 128-row tile, 8 groups of 16 rows; rows
// 16k .. 16k + 7 hold the gate rows of the tile's outputs 8k .. 8k + 7 and rows
// 16k + 8 .. 16k + 15 the matching up rows. A 16x256b TMEM load gives thread
// t of a warp lanes t/4 and t/4 + 8 of a 16-lane group at token columns
// c0 + 2 (t % 4) and + 1, i.e. a gate row and its own up row, so every thread
// finishes SiLU(g) * u for its outputs with no exchange between threads.
// Warp quarter q holds groups 2q and 2q + 1 (h = 0, 1).
// get_pairs(c0, h, v): v[0], v[1] = gate accumulators of this thread's two
// token columns, v[2], v[3] = the up accumulators (see tmem_ld_16x256b).
// Arithmetic per output: g = fp16(dequant(gate)), u = fp16(dequant(up)),
// out = fp16(silu_f16(g) * u) -- lightweight_runner.py:358 on the fp16 gate/up
// projections.
template <int NT, typename PairFn>
__device__ __forceinline__ void silu_tile(const LinearArgs& p, const float* sa, int m_tile, int n_tile, int cb,
                                          int ce, PairFn&& get_pairs) {
  const int lane = threadIdx.x & 31;
  const int q = (int)(threadIdx.x >> 5) & 3;
  const int i = lane >> 2, e2 = 2 * (lane & 3);
  float swg[2], swu[2], bg[2], bu[2];
  int rg[2], col[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    rg[h] = n_tile * kTileN + 32 * q + 16 * h + i;  // gate row; its up row is rg + 8
    col[h] = n_tile * 64 + 16 * q + 8 * h + i;      // output column
    swg[h] = p.sw[rg[h]];
    swu[h] = p.sw[rg[h] + 8];
    bg[h] = p.bias ? p.bias[rg[h]] : 0.f;
    bu[h] = p.bias ? p.bias[rg[h] + 8] : 0.f;
  }
  __half* out = static_cast<__half*>(p.out);
  for (int c0 = cb; c0 < ce; c0 += 8) {
    int32_t v[2][4];
    get_pairs(c0, 0, v[0]);
    get_pairs(c0, 1, v[1]);
    const int m0 = m_tile * NT + c0 + e2;  // this thread's tokens m0, m0 + 1
    if (p.acc_out) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int x = 0; x < 2; ++x)
          if (m0 + x < p.M) {
            p.acc_out[(size_t)(m0 + x) * p.N + rg[h]] = v[h][x];
            p.acc_out[(size_t)(m0 + x) * p.N + rg[h] + 8] = v[h][2 + x];
          }
    }
    float amax[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        const int m = m0 + x;
        if (m < p.M) {
          const float g = __half2float(__float2half_rn(dequant(v[h][x], sa[m], swg[h], p.bias, bg[h])));
          const float u = __half2float(__float2half_rn(dequant(v[h][2 + x], sa[m], swu[h], p.bias, bu[h])));
          const __half hh = __float2half_rn(__fmul_rn(silu_f16(g), u));
          out[(size_t)m * p.ld_out + col[h]] = hh;
          amax[x] = fmaxf(amax[x], fabsf(__half2float(hh)));
        }
      }
    }
    if (p.absmax_out) {
      // per token: the max over the 8 lanes that share it (same lane % 4)
#pragma unroll
      for (int x = 0; x < 2; ++x) {
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) amax[x] = fmaxf(amax[x], __shfl_xor_sync(0xffffffffu, amax[x], o));
        if (i == 0 && m0 + x < p.M) atomic_max_nonneg(p.absmax_out + m0 + x, amax[x]);
      }
    }
  }
}

// Residual epilogue of 8 token columns [c0, c0 + 8) of tile row `row`, with
// the chunk's residuals already in registers: out = fp16(fp16(v) + res).
template <int NT>
__device__ __forceinline__ void residual_chunk(const LinearArgs& p, const float* sa, int m_tile, int n_tile, int row,
                                               int c0, const int32_t (&acc)[8], const EpiOperands& e,
                                               const __half* res8) {
  const int n = n_tile * kTileN + row;
  const int m_base = m_tile * NT + c0;
  if (p.acc_out && n < p.N) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (m_base + j < p.M) p.acc_out[(size_t)(m_base + j) * p.N + n] = acc[j];
  }
  if (n >= p.N) return;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int m = m_base + j;
    if (m >= p.M) break;
    const float o = __half2float(__float2half_rn(dequant(acc[j], sa[m], e.sw, p.bias, e.bias)));
    static_cast<__half*>(p.out)[(size_t)m * p.ld_out + n] = __float2half_rn(__fadd_rn(o, __half2float(res8[j])));
  }
}

// Epilogue of a whole token tile, 8 token columns at a time; get_acc(c0, acc)
// yields the accumulators of columns [c0, c0 + 8). The residual epilogue
// loads the residuals of up to 32 tokens together before their chunks run
// (the first 8 were loaded before the accumulator was ready), so a 256-token
// prefill tile costs 8 residual round trips instead of 32. The other
// epilogues keep a compact loop.
template <int NT, typename AccFn, typename PairFn>
__device__ __forceinline__ void epilogue_tile(const LinearArgs& p, LinearCtl& c, const float* sa, int m_tile,
                                              int n_tile, int row, const EpiOperands& e, AccFn&& get_acc,
                                              PairFn&& get_pairs) {
  // this warpgroup's token columns [cb, ce)
  constexpr int kCols = NT / epi_groups_for(NT);
  const int cb = e.c_first, ce = cb + kCols;
  if (p.epilogue == NPL_EPI_SILU_MUL) {
    silu_tile<NT>(p, sa, m_tile, n_tile, cb, ce, get_pairs);
    return;
  }
  if (p.epilogue != NPL_EPI_RESIDUAL) {
    for (int c0 = cb; c0 < ce; c0 += 8) {
      int32_t acc[8];
      get_acc(c0, acc);
      epilogue_chunk<NT>(p, c, sa, m_tile, n_tile, row, c0, acc, e);
    }
    return;
  }
  constexpr int G = kCols < 32 ? kCols : 32;
  const int n = n_tile * kTileN + row;
  for (int g0 = cb; g0 < ce; g0 += G) {
    __half res[G];
#pragma unroll
    for (int j = 0; j < G; ++j) {
      if (g0 == cb && j < 8) {
        res[j] = e.res[j];
      } else {
        const int m = m_tile * NT + g0 + j;
        res[j] = (m < p.M && n < p.N) ? p.residual[(size_t)m * p.ld_res + n] : __float2half_rn(0.f);
      }
    }
#pragma unroll
    for (int cc = 0; cc < G; cc += 8) {
      int32_t acc[8];
      get_acc(g0 + cc, acc);
      residual_chunk<NT>(p, sa, m_tile, n_tile, row, g0 + cc, acc, e, res + cc);
    }
  }
}

__device__ __forceinline__ void unpack_f16x8(const uint4& x, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Activation prologue (NPL_X_F16_*), run by the 128 epilogue threads: the
// per-token scales (and RMSNorm factors), then every token tile this CTA's
// units need, quantised into shared memory in the MMA's 128-byte-swizzle
// K-major layout (unit u of the CTA uses tile slot u). Same arithmetic as
// npl_rmsnorm_quant / npl_quant_rows. Loads are issued in batches before
// their values are used, so each batch costs one memory latency.
constexpr int kRowGroup = 2;   // rows reduced together in the RMSNorm statistics
constexpr int kRowChunks = 4;  // 16-byte chunks per thread and row in flight

template <int NT>
__device__ void produce_activations(const LinearArgs& p, int8_t* xslot, float* s_scale, float* s_inv, float* s_recip,
                                    double* red,
                                    int ct) {
  const int ew = ct >> 5, lane = ct & 31;
  if (p.x_mode == NPL_X_F16_RMSNORM) {
    for (int m0 = 0; m0 < p.M; m0 += kRowGroup) {
      double ss[kRowGroup];
      float amax[kRowGroup];
#pragma unroll
      for (int r = 0; r < kRowGroup; ++r) ss[r] = 0.0;
      // pass 1: sum of squares, each row spread over all 128 threads
      for (int k0 = 0; k0 < p.K; k0 += 128 * 8 * kRowChunks) {
        uint4 buf[kRowGroup][kRowChunks];
#pragma unroll
        for (int r = 0; r < kRowGroup; ++r)
#pragma unroll
          for (int j = 0; j < kRowChunks; ++j) {
            const int k = k0 + (j * 128 + ct) * 8;
            buf[r][j] = (m0 + r < p.M && k < p.K)
                            ? *reinterpret_cast<const uint4*>(p.xf + (size_t)(m0 + r) * p.ldx + k)
                            : make_uint4(0, 0, 0, 0);
          }
#pragma unroll
        for (int r = 0; r < kRowGroup; ++r)
#pragma unroll
          for (int j = 0; j < kRowChunks; ++j) {
            float v[8];
            unpack_f16x8(buf[r][j], v);
#pragma unroll
            for (int i = 0; i < 8; ++i) ss[r] += (double)v[i] * (double)v[i];
          }
      }
#pragma unroll
      for (int r = 0; r < kRowGroup; ++r) {
        ss[r] = warp_sum(ss[r]);
        if (lane == 0) red[ew * kRowGroup + r] = ss[r];
      }
      epi_bar<NT>();
      float rr[kRowGroup];
#pragma unroll
      for (int r = 0; r < kRowGroup; ++r) {
        const double tot = red[r] + red[kRowGroup + r] + red[2 * kRowGroup + r] + red[3 * kRowGroup + r];
        const float mean = __double2float_rn(tot / (double)p.K);
        rr[r] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
        amax[r] = 0.f;
      }
      epi_bar<NT>();  // red is reused below
      // pass 2 (L1-resident rows): absmax of the normalised row
      for (int k0 = 0; k0 < p.K; k0 += 128 * 8 * kRowChunks) {
        uint4 buf[kRowGroup][kRowChunks], wbuf[kRowChunks];
#pragma unroll
        for (int j = 0; j < kRowChunks; ++j) {
          const int k = k0 + (j * 128 + ct) * 8;
          wbuf[j] = k < p.K ? *reinterpret_cast<const uint4*>(p.norm_w + k) : make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int r = 0; r < kRowGroup; ++r)
            buf[r][j] = (m0 + r < p.M && k < p.K)
                            ? *reinterpret_cast<const uint4*>(p.xf + (size_t)(m0 + r) * p.ldx + k)
                            : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < kRowChunks; ++j) {
          float w[8];
          unpack_f16x8(wbuf[j], w);
#pragma unroll
          for (int r = 0; r < kRowGroup; ++r) {
            float v[8];
            unpack_f16x8(buf[r][j], v);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float y = __half2float(__float2half_rn(__fmul_rn(v[i], rr[r])));
              amax[r] = fmaxf(amax[r], fabsf(__half2float(__float2half_rn(__fmul_rn(w[i], y)))));
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRowGroup; ++r) {
        const float a = warp_max(amax[r]);
        if (lane == 0) red[ew * kRowGroup + r] = (double)a;
      }
      epi_bar<NT>();
      if (ct < kRowGroup && m0 + ct < p.M) {
        const float a = fmaxf(fmaxf((float)red[ct], (float)red[kRowGroup + ct]),
                              fmaxf((float)red[2 * kRowGroup + ct], (float)red[3 * kRowGroup + ct]));
        s_inv[m0 + ct] = rr[ct];
        s_scale[m0 + ct] = scale_from_absmax(a);
        s_recip[m0 + ct] = quant_recip(s_scale[m0 + ct]);
      }
      epi_bar<NT>();
    }
  } else {
    for (int m = ct; m < p.M; m += 128) {
      s_scale[m] = scale_from_absmax(__int_as_float(p.x_absmax[m]));
      s_recip[m] = quant_recip(s_scale[m]);
    }
    epi_bar<NT>();
  }
  // Token tile slots: stream-K keeps one per unit of the CTA (slot u holds
  // k-block (u_begin + u) % k_blocks); cluster split-K one per k-block of the
  // CTA's range, shared by all its tiles (there is one token tile row).
  long long u_begin;
  int n_slots;
  if (p.split > 0) {
    const SplitRange r(p);
    u_begin = r.lo;
    n_slots = r.hi - r.lo;
  } else {
    u_begin = (long long)blockIdx.x * p.total_units / gridDim.x;
    n_slots = (int)((long long)(blockIdx.x + 1) * p.total_units / gridDim.x - u_begin);
  }
  const int total = n_slots * NT * 8;
  const bool norm = p.x_mode == NPL_X_F16_RMSNORM;
  constexpr int kBatch = 4;
  for (int base_item = ct; base_item < total; base_item += 128 * kBatch) {
    uint4 raw[kBatch][2], wraw[kBatch][2];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int item = base_item + b * 128;
      const int u = item / (NT * 8), r = (item >> 3) % NT, chunk = item & 7;
      const int k0 = (int)((u_begin + u) % p.k_blocks) * kBlockK + chunk * 16;
      const bool live = item < total && r < p.M && k0 < p.K;
      const __half* src = p.xf + (size_t)r * p.ldx + k0;
      raw[b][0] = live ? *reinterpret_cast<const uint4*>(src) : make_uint4(0, 0, 0, 0);
      raw[b][1] = live ? *reinterpret_cast<const uint4*>(src + 8) : make_uint4(0, 0, 0, 0);
      if (norm) {
        wraw[b][0] = live ? *reinterpret_cast<const uint4*>(p.norm_w + k0) : make_uint4(0, 0, 0, 0);
        wraw[b][1] = live ? *reinterpret_cast<const uint4*>(p.norm_w + k0 + 8) : make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int item = base_item + b * 128;
      if (item >= total) break;
      const int u = item / (NT * 8), r = (item >> 3) % NT, chunk = item & 7;
      uint4 packed = make_uint4(0, 0, 0, 0);
      if (r < p.M) {
        float v[16];
        unpack_f16x8(raw[b][0], *reinterpret_cast<float(*)[8]>(v));
        unpack_f16x8(raw[b][1], *reinterpret_cast<float(*)[8]>(v + 8));
        if (norm) {
          float w[16];
          unpack_f16x8(wraw[b][0], *reinterpret_cast<float(*)[8]>(w));
          unpack_f16x8(wraw[b][1], *reinterpret_cast<float(*)[8]>(w + 8));
          const float rr = s_inv[r];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float y = __half2float(__float2half_rn(__fmul_rn(v[i], rr)));
            v[i] = __half2float(__float2half_rn(__fmul_rn(w[i], y)));
          }
        }
        const float sc = s_scale[r], rsc = s_recip[r];
        uint32_t* w32 = reinterpret_cast<uint32_t*>(&packed);
#pragma unroll
        for (int i = 0; i < 16; ++i) w32[i >> 2] |= (uint32_t)(quantize_one(v[i], sc, rsc) & 0xff) << (8 * (i & 3));
      }
      // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
      *reinterpret_cast<uint4*>(xslot + (size_t)u * NT * kBlockK + r * kBlockK + ((chunk ^ (r & 7)) << 4)) = packed;
    }
  }
  fence_proxy_async_smem();  // the tensor cores read these tiles through the async proxy
}

__device__ __forceinline__ int ld_acquire_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// SiLU * up with silu_q: after every CTA of the grid has stored its outputs
// and their per-token absmax (a grid-wide count: every CTA of the grid is
// resident at once, since the grid has at most one CTA per SM or, under
// cluster split-K, only as many clusters as fit at once, and the next kernel
// can launch only after all of them have started), every CTA
// quantises an interleaved share of the [M, N/2] rows per token, exactly as
// npl_quant_rows would (w8a8.py:106-115), so that the down projection takes
// int8 rows without a separate quantisation launch. The last CTA done
// clears the absmax words and both counts for the next call. Run by every
// epilogue thread of the CTA.
template <int NT>
__device__ void silu_quant_rows(const LinearArgs& p, LinearCtl& c, int ct) {
  constexpr int kGroups = epi_groups_for(NT);
  constexpr int kThr = 128 * kGroups;
  epi_all_bar(kGroups);  // this CTA's outputs and absmax atomics are issued
  if (ct == 0) {
    __threadfence();
    atomicAdd(p.ws_gcnt, 1);
    const uint64_t t0 = globaltimer_ns();
    int ok = 1;
    while (ld_acquire_gpu(p.ws_gcnt) < (int)gridDim.x) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicCAS(p.status, 0, (int)NPL_DEV_TIMEOUT_EPILOGUE);
        ok = 0;
        break;
      }
    }
    c.last_flag = ok;
  }
  epi_all_bar(kGroups);
  if (!c.last_flag) return;  // the status word reports it
  const int cols = p.N / 2, chunks_per_row = cols / 8;
  const int chunks = p.M * chunks_per_row;
  __half* out = static_cast<__half*>(p.out);
  for (int i = (int)blockIdx.x * kThr + ct; i < chunks; i += (int)gridDim.x * kThr) {
    const int m = i / chunks_per_row, c0 = (i - m * chunks_per_row) * 8;
    const float sc = scale_from_absmax(__int_as_float(__ldcg(p.absmax_out + m)));
    const float rs = quant_recip(sc);
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(out + (size_t)m * p.ld_out + c0));
    const __half* h = reinterpret_cast<const __half*>(&v);
    uint2 qv;
    uint32_t* w = reinterpret_cast<uint32_t*>(&qv);
    w[0] = w[1] = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      w[e / 4] |= (uint32_t)(quantize_one(__half2float(h[e]), sc, rs) & 0xff) << (8 * (e % 4));
    *reinterpret_cast<uint2*>(p.silu_q + (size_t)m * cols + c0) = qv;
  }
  if (blockIdx.x == 0)
    for (int m = ct; m < p.M; m += kThr) p.silu_qs[m] = scale_from_absmax(__int_as_float(__ldcg(p.absmax_out + m)));
  epi_all_bar(kGroups);  // every read of the absmax words before the done count
  if (ct == 0 && atomic_add_acq_rel(p.ws_gcnt + 1, 1) + 1 == (int)gridDim.x) {
    for (int m = 0; m < p.M; ++m) atomicExch(p.absmax_out + m, 0);
    atomicExch(p.ws_gcnt, 0);
    atomicExch(p.ws_gcnt + 1, 0);
  }
}

// kXF16: the fp16-activation modes (their prologue costs registers, so the
// int8-activation kernel is compiled without it).
template <int NT, bool kXF16>
__global__ void __launch_bounds__(threads_for(NT), 1)
    w8a8_linear_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                       const LinearArgs p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                         ~uintptr_t(1023));
  LinearCtl& c = *reinterpret_cast<LinearCtl*>(base);
  int8_t* ring_a = reinterpret_cast<int8_t*>(base + p.off_a);
  int8_t* ring_b = reinterpret_cast<int8_t*>(base + p.off_b);
  int8_t* xslot = reinterpret_cast<int8_t*>(base + p.off_x);
  float* s_scale = reinterpret_cast<float*>(base + p.off_f);
  float* s_inv = s_scale + NT;
  float* s_recip = s_inv + NT;
  constexpr uint32_t kTmemCols = tmem_cols_for(NT);
  constexpr int kAccBufs = acc_bufs_for(NT);
  constexpr uint32_t kIdesc = idesc_i8(kTileN, NT);
  constexpr bool x_int8 = !kXF16;
  constexpr int kEpiGroups = epi_groups_for(NT);
  static_assert(kEpiGroups == 1 || !kXF16, "the fp16-activation prologue runs on one epilogue warpgroup");
  const uint32_t stage_bytes = kTileN * kBlockK + (x_int8 ? NT * kBlockK : 0);
  const int stages = p.stages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmap_w);
    if (x_int8) prefetch_tensormap(&tmap_x);
    for (int i = 0; i < stages; ++i) {
      mbar_init(&c.full[i], 1);
      mbar_init(&c.empty[i], 1);
    }
    for (int i = 0; i < kAccBufs; ++i) {
      mbar_init(&c.tfull[i], 1);
      mbar_init(&c.tempty[i], 4 * kEpiGroups);
    }
    mbar_init(&c.teardown, 1);
    mbar_init(&c.xready, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&c.rfull[i], 1);
      mbar_init(&c.rfree[i], 1);
    }
    fence_mbar_init();
  }
  const bool clustered = p.split > 1;
  int32_t* red = reinterpret_cast<int32_t*>(base + p.off_r);
  if (clustered) {
    // the leader's partial-tile buffers start at zero: contributors add into
    // them through the async proxy
    for (int i = threadIdx.x; i < p.red_bufs * NT * kTileN; i += (int)blockDim.x) red[i] = 0;
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(&c.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = c.tmem_base;
  // Barriers and buffers of every CTA of the cluster are initialised before
  // any CTA reaches into another (each role waits where it first needs it).
  if (clustered) {
    cluster_arrive_release();
    if (threadIdx.x != 0) cluster_wait_acquire();  // thread 0 (TMA) waits after its first weight loads
  }
  pdl_trigger();  // the next kernel may start launching its CTAs

  if (warp == 0) {
    // ---------------------------------------------------------- TMA producer
    if (lane == 0) {
      // decode tiles read each weight tile once: evict first; prefill tiles
      // read it once per token tile, so it stays in L2 for the next one
      const uint64_t pol_w = NT >= 128 ? policy_evict_normal() : policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      // Weights do not depend on earlier kernels: the weight tiles of the
      // first ring stages are requested before waiting for the previous
      // kernel; the token tiles (its output) only after. (Prefetching further
      // weight tiles into L2 here was measured slower on B200: the requests
      // delay the previous kernel's completion and this kernel's token loads.)
      int pre = 0;
      {
        SegmentIter<NT> it(p);
        int tile, kb0, kb1;
        while (pre < stages && it.next(tile, kb0, kb1)) {
          int m_tile, n_tile;
          tile_coords<NT>(p, tile, m_tile, n_tile);
          for (int kb = kb0; kb < kb1 && pre < stages; ++kb, ++pre) {
            mbar_arrive_expect_tx(&c.full[pre], stage_bytes);
            tma_load_2d(ring_a + (size_t)pre * kTileN * kBlockK, &tmap_w, kb * kBlockK, n_tile * kTileN,
                        &c.full[pre], pol_w);
          }
        }
      }
      uint32_t outstanding = (1u << pre) - 1;  // stages holding a load (pre <= 12)
      if (clustered) cluster_wait_acquire();
      pdl_wait();
      SegmentIter<NT> it(p);
      int tile, kb0, kb1, stage = 0, unit = 0;
      uint32_t phase = 0;
      bool ok = true;
      while (ok && it.next(tile, kb0, kb1)) {
        int m_tile, n_tile;
        tile_coords<NT>(p, tile, m_tile, n_tile);
        for (int kb = kb0; kb < kb1; ++kb, ++unit) {
          if (unit >= pre) {
            if (!mbar_wait(&c.empty[stage], phase ^ 1, p.status, NPL_DEV_TIMEOUT_TMA)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&c.full[stage], stage_bytes);
            tma_load_2d(ring_a + (size_t)stage * kTileN * kBlockK, &tmap_w, kb * kBlockK, n_tile * kTileN,
                        &c.full[stage], pol_w);
          }
          if (x_int8)
            tma_load_2d(ring_b + (size_t)stage * NT * kBlockK, &tmap_x, kb * kBlockK, m_tile * NT, &c.full[stage],
                        pol_x);
          outstanding |= 1u << stage;
          if (++stage == stages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every issued load must land before the CTA's shared memory is
      // released. A stage's last load used parity (phase of that issue).
      for (int i = 0; i < stages; ++i) {
        if (!(outstanding >> i & 1)) continue;
        const uint32_t par = i < stage ? phase : phase ^ 1;
        mbar_wait(&c.full[i], par, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = x_int8 || mbar_wait(&c.xready, 0, p.status, NPL_DEV_TIMEOUT_MMA);
      SegmentIter<NT> it(p);
      int tile, kb0, kb1, stage = 0, seg = 0, unit = 0;
      uint32_t phase = 0;
      while (ok && it.next(tile, kb0, kb1)) {
        const int buf = seg % kAccBufs;
        const uint32_t tphase = (seg / kAccBufs) & 1;
        if (!mbar_wait(&c.tempty[buf], tphase ^ 1, p.status, NPL_DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(buf * NT);
        for (int kb = kb0; kb < kb1; ++kb, ++unit) {
          if (!mbar_wait(&c.full[stage], phase, p.status, NPL_DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(ring_a + (size_t)stage * kTileN * kBlockK);
          const int xs = p.split > 0 ? kb - kb0 : unit;  // token tile slot (see produce_activations)
          const uint32_t b0 = x_int8 ? smem_u32(ring_b + (size_t)stage * NT * kBlockK)
                                     : smem_u32(xslot + (size_t)xs * NT * kBlockK);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 32; ++kk) {
            mma_i8(d, sdesc_k_sw128(a0 + kk * 32), sdesc_k_sw128(b0 + kk * 32), kIdesc,
                   (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&c.empty[stage]);
          if (++stage == stages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&c.tfull[buf]);
        ++seg;
      }
      // all MMAs issued by this thread complete before TMEM is freed
      tc_commit(&c.teardown);
      mbar_wait(&c.teardown, 0, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;
    const int ct = threadIdx.x - 64;  // 0 .. 128 * kEpiGroups - 1
    const int c_first = epi_group<NT>() * (NT / kEpiGroups);  // this warpgroup's first token column
    pdl_wait();
    if constexpr (kXF16) {
      produce_activations<NT>(p, xslot, s_scale, s_inv, s_recip, reinterpret_cast<double*>(s_recip + NT), ct);
      mbar_arrive(&c.xready);
      if (p.x_mode == NPL_X_F16_ABSMAX) {
        // x_absmax is consumed: the last CTA to have read it zeroes it for the
        // producer of the next call
        epi_bar<NT>();
        if (ct == 0 && atomic_add_acq_rel(p.ws_xcnt, 1) + 1 == (int)gridDim.x) {
          for (int m = 0; m < p.M; ++m) p.x_absmax[m] = 0;
          *p.ws_xcnt = 0;
        }
      }
    }
    // per-token activation scales from shared memory when there is one token
    // tile (decode); int8 activations bring theirs from global memory
    const float* sa = s_scale;
    if (x_int8) {
      if (p.M <= NT) {
        for (int m = ct; m < p.M; m += 128 * kEpiGroups) s_scale[m] = p.sa[m];
        epi_all_bar(kEpiGroups);
      } else {
        sa = p.sa;
      }
    }
    // Cluster split-K: rank 0 leads every tile of the cluster. The other
    // ranks add their partial accumulator, straight from registers, into the
    // leader's buffer in its shared memory (red.async, counted in bytes on the
    // leader's rfull barrier); the leader adds its own TMEM accumulator,
    // clears the buffer and runs the epilogue. Buffer rb is handed back to the
    // contributors (rfree) once cleared, when a later tile of the cluster
    // needs it.
    const SplitRange sr(p);
    const bool leader = sr.rank == 0;
    const uint32_t red_bytes = (uint32_t)(NT * kTileN * sizeof(int32_t));
    const int cluster_tiles =
        clustered ? (p.tiles - (int)(blockIdx.x / (unsigned)p.split) + p.clusters - 1) / p.clusters : 0;
    SegmentIter<NT> it(p);
    int tile, kb0, kb1, seg = 0;
    while (it.next(tile, kb0, kb1)) {
      const int buf = seg % kAccBufs;
      const uint32_t tphase = (seg / kAccBufs) & 1;
      int m_tile, n_tile;
      tile_coords<NT>(p, tile, m_tile, n_tile);
      const bool contributor = clustered && !leader;
      EpiOperands eo;
      if (!contributor) load_epi_operands<NT>(p, m_tile, n_tile, row, c_first, eo);
      if (!mbar_wait(&c.tfull[buf], tphase, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(buf * NT);
      if (clustered) {
        const int rb = seg % p.red_bufs, use = seg / p.red_bufs;
        int32_t* rbuf = red + (size_t)rb * NT * kTileN;  // [NT][128]: column = token, row = weight row
        if (leader) {
          if (ct == 0) mbar_arrive_expect_tx(&c.rfull[rb], (uint32_t)(p.split - 1) * red_bytes);
          mbar_wait_cluster(&c.rfull[rb], use & 1, p.status, NPL_DEV_TIMEOUT_EPILOGUE);
          epilogue_tile<NT>(
              p, c, sa, m_tile, n_tile, row, eo,
              [&](int c0, int32_t(&acc)[8]) {
                tmem_ld_x8(taddr + c0, acc);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  int32_t* cell = rbuf + (c0 + j) * kTileN + row;
                  acc[j] += *cell;  // int32 sums are exact in any order
                  *cell = 0;
                }
              },
              [&](int c0, int h, int32_t(&v)[4]) {
                tmem_ld_16x256b(taddr + ((uint32_t)(16 * h) << 16) + (uint32_t)c0, v);
                tmem_wait_ld();
                const int r = 32 * quarter + 16 * h + (lane >> 2), cc = c0 + 2 * (lane & 3);
#pragma unroll
                for (int k = 0; k < 4; ++k) {  // (gate, up) x (cc, cc + 1); rows of this warp's quarter
                  int32_t* cell = rbuf + (cc + (k & 1)) * kTileN + r + 8 * (k >> 1);
                  v[k] += *cell;
                  *cell = 0;
                }
              });
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&c.tempty[buf]);
          if (seg + p.red_bufs < cluster_tiles) {
            fence_proxy_async_smem();  // the cleared cells, before the contributors' next adds
            epi_bar<NT>();
            if (ct > 0 && ct < p.split) mbar_arrive_remote(cluster_map(&c.rfree[rb], (uint32_t)ct));
          }
        } else {
          if (seg >= p.red_bufs) mbar_wait_cluster(&c.rfree[rb], (use - 1) & 1, p.status, NPL_DEV_TIMEOUT_EPILOGUE);
          const uint32_t dst = cluster_map(rbuf + row, 0);
          const uint32_t bar = cluster_map(&c.rfull[rb], 0);
          for (int c0 = 0; c0 < NT; c0 += 8) {
            int32_t acc[8];
            tmem_ld_x8(taddr + c0, acc);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j)
              red_add_s32_cluster(dst + (uint32_t)((c0 + j) * kTileN * sizeof(int32_t)), acc[j], bar);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&c.tempty[buf]);
        }
        ++seg;
        continue;
      }
      const bool whole = (kb0 == 0 && kb1 == p.k_blocks);
      // a partial tile lies in the stream-K range: slot = (first CTA boundary
      // strictly inside the tile, counted in that range's units) - 1
      int slot = 0;
      if (!whole) {
        const long long first_unit = (long long)(tile - p.dp_tiles) * p.k_blocks;
        slot = (int)(((first_unit + 1) * gridDim.x + p.sk_units - 1) / p.sk_units) - 1;
      }
      int32_t* ws = p.ws_acc + (size_t)slot * NT * kTileN;
      if (whole) {
        epilogue_tile<NT>(
            p, c, sa, m_tile, n_tile, row, eo,
            [&](int c0, int32_t(&acc)[8]) {
              tmem_ld_x8(taddr + c0, acc);
              tmem_wait_ld();
            },
            [&](int c0, int h, int32_t(&v)[4]) {
              tmem_ld_16x256b(taddr + ((uint32_t)(16 * h) << 16) + (uint32_t)c0, v);
              tmem_wait_ld();
            });
      } else {
        for (int c0 = c_first; c0 < c_first + NT / kEpiGroups; c0 += 8) {
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
      if (lane == 0) mbar_arrive(&c.tempty[buf]);
      if (!whole) {
        epi_all_bar(kEpiGroups);  // every warpgroup's adds before the count
        if (ct == 0) c.last_flag = (atomic_add_acq_rel(p.ws_cnt + slot, kb1 - kb0) + (kb1 - kb0) == p.k_blocks);
        epi_all_bar(kEpiGroups);
        if (c.last_flag) {
          epilogue_tile<NT>(
              p, c, sa, m_tile, n_tile, row, eo,
              [&](int c0, int32_t(&acc)[8]) {
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  int32_t* cell = ws + (size_t)(c0 + j) * kTileN + row;
                  acc[j] = __ldcg(cell);
                  __stcg(cell, 0);
                }
              },
              [&](int c0, int h, int32_t(&v)[4]) {
                const int r = 32 * quarter + 16 * h + (lane >> 2), cc = c0 + 2 * (lane & 3);
#pragma unroll
                for (int k = 0; k < 4; ++k) {  // (gate, up) x (cc, cc + 1)
                  int32_t* cell = ws + (size_t)(cc + (k & 1)) * kTileN + r + 8 * (k >> 1);
                  v[k] = __ldcg(cell);
                  __stcg(cell, 0);
                }
              });
          if (ct == 0) p.ws_cnt[slot] = 0;
        }
        epi_all_bar(kEpiGroups);  // last_flag is read before the next tile sets it
      }
      ++seg;
    }
    if (p.silu_q) silu_quant_rows<NT>(p, c, ct);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  // No CTA of a cluster waits for the others at exit: the leader's buffers
  // and barriers are last written by the adds its final rfull wait counted,
  // and a contributor's barriers are only signalled while it waits on them.
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

// Workspace: grid - 1 partial-tile slots of NT x 128 int32, one counter per
// slot and one activation-reader counter; grid <= number of SMs of the
// current device.
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
  return ws_acc_bytes(M) + (((slots + 3) * sizeof(int32_t) + 255) & ~size_t(255));
}

constexpr uint32_t align1k(size_t x) { return (uint32_t)((x + 1023) & ~size_t(1023)); }

// Clusters of `split` CTAs of `kern` with `smem` bytes that fit on the
// device at once (cached per device, kernel, shared memory and size).
int max_active_clusters(const void* kern, int smem, int split, int block) {
  struct Entry {
    int dev;
    const void* kern;
    int smem, split, n;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : cache)
    if (e.dev == dev && e.kern == kern && e.smem == smem && e.split == split) return e.n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)split);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)split;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  cache.push_back({dev, kern, smem, split, n});
  return n;
}

// Shared memory that leaves room for one CTA per SM only: the cluster
// capacity at this size is the number of clusters that fit with every CTA on
// an SM of its own. (GPCs differ in size, so on B200 clusters of 3 or 4 fit
// on fewer than all 148 SMs: placing more doubles CTAs up on some SMs.)
constexpr int kOnePerSmSmem = 120 * 1024;

struct Schedule {
  int split;     // 0: stream-K; >= 1: CTAs per tile (cluster size)
  int clusters;  // cluster split-K: clusters in the grid
};

// Decode tiles: cluster split-K with S CTAs per tile (S <= 8) and C clusters
// (C <= the clusters that fit one CTA per SM), or stream-K over all SMs,
// whichever has the least per-CTA work in (tile, k-block) units. Stream-K's
// global partial-tile reduction costs about 3 units more than the DSMEM one
// (measured on B200: ~1 us against 0.35 us per 16 KB weight unit).
constexpr int kStreamKFixupUnits = 3;

Schedule pick_schedule(const void* kern, int block, int tiles, int k_blocks, long long units, int grid_max) {
  Schedule best{0, 0};
  long long best_cost = (units + grid_max - 1) / grid_max + kStreamKFixupUnits;
  for (int s = 1; s <= 8 && s <= k_blocks; ++s) {
    const int cap = s == 1 ? grid_max : max_active_clusters(kern, kOnePerSmSmem, s, block);
    const int c = std::min(tiles, std::min(cap, grid_max / s));
    if (c < 1) continue;
    const long long cost = (long long)((tiles + c - 1) / c) * ((k_blocks + s - 1) / s);
    if (cost < best_cost) {
      best_cost = cost;
      best = {s, c};
    }
  }
  return best;
}

// Shared-memory layout for the schedule in `p` (split, x_slots); returns the
// dynamic shared memory size, or 0 when the stage ring does not fit.
template <int NT>
int layout_linear(LinearArgs& p) {
  const bool x_int8 = p.x_mode == NPL_X_INT8;
  const size_t stage_bytes = (size_t)kTileN * kBlockK + (x_int8 ? (size_t)NT * kBlockK : 0);
  const size_t xslots = x_int8 ? 0 : (size_t)p.x_slots * NT * kBlockK;
  const size_t reds = (size_t)p.red_bufs * NT * kTileN * sizeof(int32_t);
  const size_t tail = 3 * NT * sizeof(float) + 8 * sizeof(double);
  p.off_a = align1k(sizeof(LinearCtl));
  // Decode tiles (NT <= 64) keep the CTA near 110 KB when they can, so that
  // the next kernel's CTA fits beside it on an SM and starts its weight loads
  // while this one finishes; prefill tiles take the whole shared memory.
  const size_t fixed = p.off_a + xslots + reds + tail + 1024 + 1024;
  int stages = 0;
  if (NT <= 64 && fixed + 3 * stage_bytes <= (size_t)kCoresidentSmem)
    stages = (int)std::min<size_t>(6, (kCoresidentSmem - fixed) / stage_bytes);
  else if (fixed + 2 * stage_bytes <= (size_t)kMaxSmem)
    stages = (int)std::min<size_t>(kMaxStages, (kMaxSmem - fixed) / stage_bytes);
  if (stages < 2) return 0;
  p.stages = stages;
  p.off_b = p.off_a + (uint32_t)(stages * kTileN * kBlockK);
  p.off_x = p.off_b + (uint32_t)(x_int8 ? stages * NT * kBlockK : 0);
  p.off_r = p.off_x + (uint32_t)xslots;  // 1 KB aligned: stage and slot sizes are multiples of 1 KB
  p.off_f = p.off_r + (uint32_t)reds;
  return (int)(p.off_f + tail + 1024);
}

// Token tiles per raster group of the prefill tile numbering (tile_coords):
// the ~148 tiles in flight then share 8 token tiles (8 x 256 rows of
// activations) and ~18 weight tiles, read from DRAM once per wave.
constexpr int kRasterGroup = 8;

template <int NT>
int launch_linear(const CUtensorMap& tw, const CUtensorMap& tx, LinearArgs& p, cudaStream_t st) {
  const bool x_int8 = p.x_mode == NPL_X_INT8;
  void (*kern)(CUtensorMap, CUtensorMap, LinearArgs);
  if constexpr (NT > 64) {
    if (!x_int8) return fail(NPL_ERR_UNSUPPORTED, "npl_w8a8_linear: fp16 activations take at most 64 tokens");
    kern = w8a8_linear_kernel<NT, false>;
  } else {
    kern = x_int8 ? w8a8_linear_kernel<NT, false> : w8a8_linear_kernel<NT, true>;
  }
  p.raster_g = 1;
  p.dp_tiles = 0;
  p.sk_units = p.total_units;
  const int grid_max = max_grid();
  const void* kfn = reinterpret_cast<const void*>(kern);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess)
    return launch_status("npl_w8a8_linear: smem attribute");
  int smem = 0, grid = 0;
  if (NT <= 64) {
    const Schedule s = pick_schedule(kfn, threads_for(NT), p.tiles, p.k_blocks, p.total_units, grid_max);
    if (s.split > 0) {
      p.split = s.split;
      p.clusters = s.clusters;
      p.red_bufs = s.split > 1 ? (NT <= 16 ? 2 : 1) : 0;
      p.x_slots = (p.k_blocks + s.split - 1) / s.split;
      smem = layout_linear<NT>(p);
      // the schedule has no second wave: all clusters must be resident at once
      if (smem && p.split > 1 && max_active_clusters(kfn, smem, p.split, threads_for(NT)) < p.clusters) smem = 0;
      grid = p.clusters * p.split;
    }
  }
  if (!smem) {  // stream-K
    p.split = p.clusters = p.red_bufs = 0;
    grid = (int)std::min<long long>(grid_max, p.total_units);
    if (NT >= 128) {
      // prefill: grouped tile numbering, whole tiles (one per CTA per wave,
      // no partial-tile fix-up). With three or more waves every tile runs
      // whole: a ragged last wave costs less than stream-K's partial tiles,
      // whose int32 fix-up moves 128 KB of atomics per contribution (config-4
      // GEMMs on one B200: 1250-1282 us all whole against 1371-1442 with the
      // last one to two waves split). Two waves: the second is split evenly
      // by stream-K; fewer tiles than SMs: stream-K over all of them.
      p.raster_g = std::min(kRasterGroup, p.tiles / p.n_tiles);
      const int waves = p.tiles / grid;
      if (waves >= 3) p.dp_tiles = p.tiles;
      else if (waves == 2) p.dp_tiles = grid;
      p.sk_units = p.total_units - (long long)p.dp_tiles * p.k_blocks;
    }
    p.x_slots = (int)((p.total_units + grid - 1) / grid);
    smem = layout_linear<NT>(p);
    if (!smem)
      return fail(NPL_ERR_UNSUPPORTED, "npl_w8a8_linear: %d fp16 token tiles do not fit in shared memory",
                  p.x_slots);
  }
  return launch_pdl_cluster("npl_w8a8_linear", kern, dim3((unsigned)grid), dim3(threads_for(NT)), (size_t)smem, st,
                            (unsigned)std::max(p.split, 1), tw, tx, p);
}

struct LinearCall {
  const int8_t* qa;
  int lda;
  const float* sa;
  const void* xf;
  int ldx;
  int32_t* x_absmax;
  const void* norm_w;
  float eps;
  int x_mode;
  const int8_t* qw;
  int ldw;
  const float* sw;
  const float* bias;
  int M, N, K;
  int epilogue;
  const void* residual;
  int ld_res;
  void* out;
  int ld_out;
  int out_dtype;
  int32_t* acc_out;
  int32_t* absmax_out;
  const npl_rope_kv* rope;
  int8_t* silu_q;
  float* silu_qs;
};

int run_linear(const LinearCall& a, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_device()) return rc;
  const int M = a.M, N = a.N, K = a.K;
  if (!a.qw || !a.sw) return fail(NPL_ERR_ARG, "npl_w8a8_linear: null weight or weight scales");
  if (M < 0 || N <= 0 || K <= 0 || K % 16 || a.ldw < K || a.ldw % 16)
    return fail(NPL_ERR_ARG, "npl_w8a8_linear: bad shape M=%d N=%d K=%d ldw=%d", M, N, K, a.ldw);
  if ((long long)K * 127 * 127 >= (1ll << 31))
    return fail(NPL_ERR_OVERFLOW, "npl_w8a8_linear: worst-case dot product exceeds signed INT32 (K=%d)", K);
  if (!aligned16(a.qw)) return fail(NPL_ERR_ARG, "npl_w8a8_linear: int8 weights must be 16-byte aligned");
  if (a.x_mode == NPL_X_INT8) {
    if (!a.qa || !a.sa || a.lda < K || a.lda % 16 || !aligned16(a.qa))
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: int8 activations need qa/sa, lda >= K, lda %% 16 == 0, 16-B alignment");
  } else if (a.x_mode == NPL_X_F16_ABSMAX || a.x_mode == NPL_X_F16_RMSNORM) {
    if (!a.xf || a.ldx < K || a.ldx % 8 || !aligned16(a.xf))
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: fp16 activations need x, ldx >= K, ldx %% 8 == 0, 16-B alignment");
    if (M > 64) return fail(NPL_ERR_UNSUPPORTED, "npl_w8a8_linear: fp16 activations take at most 64 tokens");
    if (a.x_mode == NPL_X_F16_ABSMAX && !a.x_absmax)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: NPL_X_F16_ABSMAX needs the per-token absmax");
    if (a.x_mode == NPL_X_F16_RMSNORM && (!a.norm_w || !aligned16(a.norm_w)))
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: NPL_X_F16_RMSNORM needs a 16-B aligned norm weight");
  } else {
    return fail(NPL_ERR_ARG, "npl_w8a8_linear: unknown activation mode %d", a.x_mode);
  }
  if (a.epilogue == NPL_EPI_RESIDUAL) {
    if (!a.out || !a.residual || a.out_dtype != NPL_F16 || a.ld_res < N || a.ld_out < N)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: residual epilogue needs fp16 residual/out with ld >= N");
  } else if (a.epilogue == NPL_EPI_SILU_MUL) {
    if (!a.out || N % kTileN || a.out_dtype != NPL_F16 || a.ld_out < N / 2)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: SiLU*up epilogue needs N %% 128 == 0, fp16 out, ld_out >= N/2");
    if (a.silu_q && (!a.silu_qs || !a.absmax_out || M > 64 || a.ld_out % 8 || !aligned16(a.out) ||
                     (reinterpret_cast<uintptr_t>(a.silu_q) & 7u)))
      return fail(NPL_ERR_ARG,
                  "npl_w8a8_linear: q_out needs q_scale, absmax_out, M <= 64, ld_out %% 8 == 0, a 16-byte aligned "
                  "out and an 8-byte aligned q_out");
  } else if (a.epilogue == NPL_EPI_NONE) {
    if (!a.out || (a.out_dtype != NPL_F16 && a.out_dtype != NPL_F32) || a.ld_out < N)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: out_dtype must be NPL_F16/NPL_F32 and ld_out >= N");
  } else if (a.epilogue == NPL_EPI_ROPE_KV) {
    const npl_rope_kv* r = a.rope;
    if (!r || !r->cos_table || !r->sin_table || !r->positions || !r->slot_mapping || !r->q_out || !r->k_cache ||
        !r->v_cache)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: RoPE epilogue needs tables, positions, slots, q_out and caches");
    const int D = r->head_dim;
    if (D <= 0 || D % 2 || kTileN % D || (r->heads * D) % kTileN || (r->kv_heads * D) % kTileN ||
        r->heads % r->kv_heads || N != (r->heads + 2 * r->kv_heads) * D || r->max_position <= 0 ||
        r->num_blocks <= 0 || r->block_size <= 0)
      return fail(NPL_ERR_ARG, "npl_w8a8_linear: RoPE epilogue geometry (N = (H + 2 Hkv) D, head blocks of 128)");
  } else {
    return fail(NPL_ERR_ARG, "npl_w8a8_linear: unknown epilogue %d", a.epilogue);
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
  p.x_mode = a.x_mode;
  p.sa = a.sa;
  p.xf = static_cast<const __half*>(a.xf);
  p.ldx = a.ldx;
  p.x_absmax = a.x_absmax;
  p.norm_w = static_cast<const __half*>(a.norm_w);
  p.eps = a.eps;
  p.sw = a.sw;
  p.bias = a.bias;
  p.epilogue = a.epilogue;
  p.residual = static_cast<const __half*>(a.residual);
  p.ld_res = a.ld_res;
  p.out = a.out;
  p.ld_out = a.ld_out;
  p.out_dtype = a.out_dtype;
  p.acc_out = a.acc_out;
  p.absmax_out = a.absmax_out;
  p.silu_q = a.silu_q;
  p.silu_qs = a.silu_qs;
  if (a.epilogue == NPL_EPI_ROPE_KV) {
    const npl_rope_kv* r = a.rope;
    p.cos_t = static_cast<const __half*>(r->cos_table);
    p.sin_t = static_cast<const __half*>(r->sin_table);
    p.max_position = r->max_position;
    p.positions = r->positions;
    p.slots = r->slot_mapping;
    p.q_out = static_cast<__half*>(r->q_out);
    p.k_cache = static_cast<__half*>(r->k_cache);
    p.v_cache = static_cast<__half*>(r->v_cache);
    p.num_slots = (long long)r->num_blocks * r->block_size;
    p.heads = r->heads;
    p.kv_heads = r->kv_heads;
    p.head_dim = r->head_dim;
  }
  p.ws_acc = static_cast<int32_t*>(workspace);
  p.ws_cnt = reinterpret_cast<int32_t*>(static_cast<char*>(workspace) + ws_acc_bytes(M));
  p.ws_xcnt = p.ws_cnt + std::max(1, max_grid() - 1);
  p.ws_gcnt = p.ws_xcnt + 1;
  p.n_tiles = (N + kTileN - 1) / kTileN;
  p.k_blocks = (K + kBlockK - 1) / kBlockK;
  const int m_tiles = (M + nt - 1) / nt;
  p.total_units = (long long)p.n_tiles * m_tiles * p.k_blocks;
  p.tiles = p.n_tiles * m_tiles;
  p.status = device_status_ptr();

  CUtensorMap tw, tx;
  if (int rc = make_map(&tw, a.qw, N, K, a.ldw, kTileN)) return rc;
  if (a.x_mode == NPL_X_INT8) {
    if (int rc = make_map(&tx, a.qa, M, K, a.lda, nt)) return rc;
  } else {
    tx = tw;  // unused
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (nt) {
    case 8: return launch_linear<8>(tw, tx, p, st);
    case 16: return launch_linear<16>(tw, tx, p, st);
    case 32: return launch_linear<32>(tw, tx, p, st);
    case 64: return launch_linear<64>(tw, tx, p, st);
    case 128: return launch_linear<128>(tw, tx, p, st);
    default: return launch_linear<256>(tw, tx, p, st);
  }
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
  if (epilogue != NPL_EPI_NONE && epilogue != NPL_EPI_RESIDUAL && epilogue != NPL_EPI_SILU_MUL)
    return fail(NPL_ERR_ARG, "npl_w8a8_linear: epilogue %d (NONE, RESIDUAL or SILU_MUL; see npl_w8a8_linear_ex)",
                epilogue);
  if (!qa || !sa || !out) return fail(NPL_ERR_ARG, "npl_w8a8_linear: null pointer");
  LinearCall a{};
  a.qa = qa;
  a.lda = lda;
  a.sa = sa;
  a.x_mode = NPL_X_INT8;
  a.qw = qw;
  a.ldw = ldw;
  a.sw = sw;
  a.bias = bias;
  a.M = M;
  a.N = N;
  a.K = K;
  a.epilogue = epilogue;
  a.residual = residual;
  a.ld_res = ld_res;
  a.out = out;
  a.ld_out = ld_out;
  a.out_dtype = out_dtype;
  a.acc_out = acc_out;
  return run_linear(a, workspace, workspace_bytes, stream);
}

extern "C" int npl_w8a8_linear_ex(const npl_linear_args* args, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  if (!args) return fail(NPL_ERR_ARG, "npl_w8a8_linear_ex: null args");
  LinearCall a{};
  a.qa = args->qa;
  a.lda = args->lda;
  a.sa = args->sa;
  a.xf = args->x_f16;
  a.ldx = args->ldx;
  a.x_absmax = args->x_absmax;
  a.norm_w = args->norm_weight;
  a.eps = args->eps;
  a.x_mode = args->x_mode;
  a.qw = args->qw;
  a.ldw = args->ldw;
  a.sw = args->sw;
  a.bias = args->bias;
  a.M = args->M;
  a.N = args->N;
  a.K = args->K;
  a.epilogue = args->epilogue;
  a.residual = args->residual;
  a.ld_res = args->ld_res;
  a.out = args->out;
  a.ld_out = args->ld_out;
  a.out_dtype = args->out_dtype;
  a.acc_out = args->acc_out;
  a.absmax_out = args->absmax_out;
  a.rope = &args->rope;
  a.silu_q = args->q_out;
  a.silu_qs = args->q_scale;
  return run_linear(a, workspace, workspace_bytes, stream);
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
// Every call outside stream capture looks up the array's device address with
// cudaGetSymbolAddress (with the device current); a call during capture uses
// the address of the device's last lookup, so make the first call on each
// device before starting any stream capture. Clearing the scratch is one
// cudaMemsetAsync of ws_bytes(M) (at most ~5 MiB at M = 64) on the caller's
// stream per call, a launch of its own ahead of the linear.
// ----------------------------------------------------------------------------
namespace npl {
namespace {

constexpr int kNoAllocMaxTokens = 64;
constexpr int kNoAllocMaxSlots = 159;  // grid - 1 for devices with up to 160 SMs
constexpr size_t kNoAllocAccBytes = (size_t)kNoAllocMaxSlots * kNoAllocMaxTokens * kTileN * sizeof(int32_t);
constexpr size_t kNoAllocBytes = kNoAllocAccBytes + ((kNoAllocMaxSlots * sizeof(int32_t) + 255) & ~size_t(255));

static __device__ __align__(256) unsigned char g_linear_scratch[kNoAllocBytes];

constexpr int kNoAllocDevices = 64;
std::atomic<void*> g_scratch_ptr[kNoAllocDevices];

// Device address of g_linear_scratch on the current device. Outside stream
// capture it is looked up on every call (cudaGetSymbolAddress is a host-side
// query, and a fresh lookup stays right after a device reset reloads the
// module); during capture the address of the last lookup on this device is
// used, so a device's first call must come before any capture. The cache
// entries are atomic: host threads may call concurrently.
int scratch_address(cudaStream_t stream, void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocDevices)
    return fail(NPL_ERR_LAUNCH, "npl_w8a8_linear_noalloc: no usable current device");
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess)
    return launch_status("npl_w8a8_linear_noalloc: stream capture status");
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
    if (e != cudaSuccess || !p)
      return fail(NPL_ERR_LAUNCH, "npl_w8a8_linear_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_scratch_ptr[dev].store(p, std::memory_order_release);
  }
  *out = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!*out)
    return fail(NPL_ERR_ARG, "npl_w8a8_linear_noalloc: the first call on a device must come before stream capture");
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
  if (int rc = npl::scratch_address(static_cast<cudaStream_t>(stream), &scratch)) return rc;
  if (cudaMemsetAsync(scratch, 0, need, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return launch_status("npl_w8a8_linear_noalloc: clearing the scratch");
  return npl_w8a8_linear(qa, lda, sa, qw, ldw, sw, bias, M, N, K, epilogue, residual, ld_res, out, ld_out,
                         out_dtype, acc_out, scratch, need, stream);
}
