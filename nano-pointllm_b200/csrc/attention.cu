// KV-cache writes (with RoPE) and decode-only paged attention.
//
// npl_store_kv               <- paged_attention.py:332-383 (store_kvcache)
// npl_rope_store_kv          <- paged_attention.py:1284-1294 (rotary_fn on q/k of
//                               the packed QKV output, then store_kvcache)
// npl_paged_decode_attention <- paged_attention.py:682-843,872-1030
//                               (split-KV tile kernel + reduce, q_len = 1)
//
// KV pool layout (kv_pool.py:9-24): one fp16 tensor per layer and K/V,
// [num_blocks, block_size, Hkv, D]; slot s lives at block s / block_size,
// offset s % block_size; block tables map a sequence's logical blocks to
// physical ones.
#include <algorithm>
#include <initializer_list>

#include <cudaTypedefs.h>

#include "npl_common.cuh"

namespace npl {
namespace {

constexpr int kDevBadIndex = NPL_DEV_BAD_INDEX;

__device__ __forceinline__ void flag_bad_index(int* status) {
  if (status) atomicCAS(status, 0, kDevBadIndex);
}

// ------------------------------------------------------------ store_kvcache
__global__ void store_kv_kernel(const __half* __restrict__ key, const __half* __restrict__ value, int ld_tok,
                                int hkv_d, const int32_t* __restrict__ slots, __half* __restrict__ kc,
                                __half* __restrict__ vc, long long num_slots, int* status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const long long slot = slots[t];
  if (slot < 0) return;  // padding token
  if (slot >= num_slots) {
    if (threadIdx.x == 0) flag_bad_index(status);
    return;
  }
  const uint4* ks = reinterpret_cast<const uint4*>(key + (size_t)t * ld_tok);
  const uint4* vs = reinterpret_cast<const uint4*>(value + (size_t)t * ld_tok);
  uint4* kd = reinterpret_cast<uint4*>(kc + slot * hkv_d);
  uint4* vd = reinterpret_cast<uint4*>(vc + slot * hkv_d);
  for (int i = threadIdx.x; i < hkv_d / 8; i += blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

// -------------------------------------------------------- RoPE + store
// Grid (token, group of `hpc` heads of q | k | v); the CTA's threads walk the
// (head, d) pairs of its group. Decode batches take one head per CTA and D/2
// threads (many small CTAs in parallel); prefill batches take every head of a
// token in one CTA (a CTA per (token, head) made ~10^6 tiny CTAs, bound by
// CTA launch). Pair (d, d + D/2) of a q/k head:
//   out[d]       = fp16(fp16(x1 * cos[d])       + fp16(-x2 * sin[d]))
//   out[d + D/2] = fp16(fp16(x2 * cos[d + D/2]) + fp16( x1 * sin[d + D/2]))
// (HF apply_rotary_pos_emb with rotate_half(x) = cat(-x2, x1), each torch
// fp16 op rounded once); v heads are copied to the cache unchanged.
__global__ void rope_store_kernel(const __half* __restrict__ qkv, int ld_qkv, int H, int Hkv, int D,
                                  const __half* __restrict__ cos_t, const __half* __restrict__ sin_t,
                                  int max_position, const int64_t* __restrict__ positions,
                                  const int32_t* __restrict__ slots, __half* __restrict__ q_out,
                                  __half* __restrict__ kc, __half* __restrict__ vc, long long num_slots,
                                  int hpc, int* status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, head0 = blockIdx.y * hpc;
  const int half_d = D / 2;
  const long long pos = positions[t];
  const long long slot = slots[t];
  const bool pos_ok = pos >= 0 && pos < max_position;
  const bool slot_ok = slot >= 0 && slot < num_slots;
  if (head0 == 0 && threadIdx.x == 0 && (!pos_ok || slot >= num_slots)) flag_bad_index(status);
  const int heads = min(hpc, H + 2 * Hkv - head0);
  for (int i = threadIdx.x; i < heads * half_d; i += blockDim.x) {
    const int head = head0 + i / half_d, d = i % half_d;
    const __half* x = qkv + (size_t)t * ld_qkv + (size_t)head * D;
    if (head >= H + Hkv) {  // v
      if (slot_ok) {
        __half* vd = vc + (slot * Hkv + (head - H - Hkv)) * D;
        vd[d] = x[d];
        vd[d + half_d] = x[d + half_d];
      }
      continue;
    }
    if (!pos_ok) continue;
    const __half* c = cos_t + pos * D;
    const __half* s = sin_t + pos * D;
    const float x1 = __half2float(x[d]);
    const float x2 = __half2float(x[d + half_d]);
    const float a1 = __half2float(__float2half_rn(__fmul_rn(x1, __half2float(c[d]))));
    const float b1 = __half2float(__float2half_rn(__fmul_rn(-x2, __half2float(s[d]))));
    const float a2 = __half2float(__float2half_rn(__fmul_rn(x2, __half2float(c[d + half_d]))));
    const float b2 = __half2float(__float2half_rn(__fmul_rn(x1, __half2float(s[d + half_d]))));
    const __half o1 = __float2half_rn(__fadd_rn(a1, b1));
    const __half o2 = __float2half_rn(__fadd_rn(a2, b2));
    __half* dst;
    if (head < H) {
      dst = q_out + ((size_t)t * H + head) * D;
    } else {
      if (!slot_ok) continue;
      dst = kc + (slot * Hkv + (head - H)) * D;
    }
    dst[d] = o1;
    dst[d + half_d] = o2;
  }
}

// ------------------------------------------------- paged decode attention
// Persistent kernel, 3 CTAs per SM, 160 threads:
//   warp 0     producer: takes work items (the CTA's first item is blockIdx.x,
//              later ones come from a global counter), looks up the block
//              table and streams the item's K and V through a ring of
//              64-token stages with TMA (3-D tensor maps over the cache viewed
//              as [tokens][Hkv][D]; one box = min(64, block_size) tokens of
//              one head)
//   warps 1-4  consumers: D/8 lanes per token, 128/(D/8) token streams, each
//              with its own online-softmax state over the item's tokens
// A work item is (chunk of the context, sequence b, head h); items are
// numbered chunk-major, so at any time the CTAs read the same token rows of
// many heads (adjacent 256-byte pieces of each 8 KB cache row), which keeps
// the DRAM accesses local. At the end of an item the streams are merged into
// a partial (max, sum, acc[D]); chunks before the last one of (b, h) publish
// theirs behind a per-chunk flag, and the item of the last chunk (which waits
// for the flags and clears them) merges them into out[b, h].
// With q_out given, the CTA that completes the last head of b quantises the
// attention row of b per token (w8a8.py:106-115), which is the input of the O
// projection.
// 3 CTAs x ~69 KB per SM (64-token stages, 2-stage rings): measured the
// fastest split on B200 (2 CTAs x 3 stages and 32-token stages were slower).
constexpr int kAttnTok = 64;
constexpr int kAttnStages = 2;
constexpr int kAttnCtasPerSm = 3;
constexpr int kAttnChunk = 256;
constexpr int kAttnMaxBatch = 1024;  // sequences per call (one counter each in the workspace)
constexpr int kAttnConsumers = 128;
constexpr int kAttnThreads = 32 + kAttnConsumers;
constexpr float kNegBig = -1.0e30f;

template <int D>
struct alignas(128) AttnSmem {
  static constexpr int kStreams = kAttnConsumers / (D / 8);
  __half k[kAttnStages][kAttnTok * D];
  __half v[kAttnStages][kAttnTok * D];
  __half q[kAttnStages][D];  // the item's query, sent with its first stage
  float acc[kStreams][D];
  float m[kStreams];
  float l[kStreams];
  float red[4];
  uint64_t full[kAttnStages];
  uint64_t empty[kAttnStages];
  int4 meta[kAttnStages];  // item (-1: no more work), stage in item, valid tokens, last stage of item
  int last_row;
};

struct AttnArgs {
  const __half* q;
  int B, H, Hkv;
  int num_blocks, block_size, box_tok;
  const int32_t* bt;
  int bt_stride, max_blocks;
  const int32_t* ctx_lens;
  float scale;
  int n_chunks, n_items;
  __half* out;
  int8_t* q_out;
  float* q_scale;
  float* part_ml;     // [B*H*n_chunks][2]
  float* part_acc;    // [B*H*n_chunks][D]
  uint32_t* flags;    // [B*H*n_chunks]: 1 once the chunk's partial is written (cleared by its owner)
  int32_t* cnt_row;   // [B]
  int32_t* work;      // [2]: next item beyond the first grid.x, CTAs done
  int* status;
};

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// 1-D bulk copy global -> shared, completion counted on `bar` (16-byte multiple).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Counter increment with acquire-release semantics at GPU scope: the CTA's
// earlier writes (ordered before this thread by a barrier) are visible to
// whoever observes the new value, and writes observed here are visible after.
__device__ __forceinline__ int atomic_add_acq_rel(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void store_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int attn_ctx(const AttnArgs& p, int b) {
  return min(max(0, p.ctx_lens[b]), p.max_blocks * p.block_size);
}

__device__ __forceinline__ void unpack8(const uint4& x, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// End of an item: the token streams are merged into the chunk's partial
// (max, sum, acc[D]). A chunk other than the last one of (b, h) publishes its
// partial and raises its flag (no round trip: the consumers go straight on).
// The last chunk owns (b, h): it waits for the earlier chunks' flags (those
// items were taken from the queue before it), merges their partials in chunk
// order and writes out[b, h].
template <int D>
__device__ void attn_item_end(const AttnArgs& p, AttnSmem<D>& s, int ct, int stream, int sl, int b, int h, int chunk,
                              float m, float l, const float (&acc)[8]) {
  constexpr int S = AttnSmem<D>::kStreams;
  const int bh = b * p.H + h;
#pragma unroll
  for (int i = 0; i < 8; ++i) s.acc[stream][sl * 8 + i] = acc[i];
  if (sl == 0) {
    s.m[stream] = m;
    s.l[stream] = l;
  }
  consumer_bar();
  float mm = kNegBig, ll = 0.f, aa = 0.f;
  if (ct < D) {
#pragma unroll
    for (int i = 0; i < S; ++i) mm = fmaxf(mm, s.m[i]);
#pragma unroll
    for (int i = 0; i < S; ++i) {
      const float w = exp2f(s.m[i] - mm);
      ll += s.l[i] * w;
      aa += s.acc[i][ct] * w;
    }
  }
  const int active = max(1, (attn_ctx(p, b) + kAttnChunk - 1) / kAttnChunk);
  const size_t pbase = (size_t)bh * p.n_chunks;
  if (chunk < active - 1) {
    if (ct < D) {
      __stcg(p.part_acc + (pbase + chunk) * D + ct, aa);
      if (ct == 0) {
        __stcg(p.part_ml + (pbase + chunk) * 2, mm);
        __stcg(p.part_ml + (pbase + chunk) * 2 + 1, ll);
      }
    }
    consumer_bar();  // every partial write is ordered before the flag (cumulative release)
    if (ct == 0) store_release(p.flags + pbase + chunk, 1u);
    consumer_bar();  // stream state in shared memory is free for the next item
    return;
  }
  if (ct == 0) {
    // wait for the earlier chunks' flags and clear each one once seen: no
    // later item of this launch sets it again, so flags are zero between calls
    for (int c = 0; c < active - 1; ++c) {
      if (load_acquire(p.flags + pbase + c) == 0u) {
        const uint64_t t0 = globaltimer_ns();
        while (load_acquire(p.flags + pbase + c) == 0u) {
          if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicCAS(p.status, 0, NPL_DEV_TIMEOUT_EPILOGUE);
            break;
          }
        }
      }
      p.flags[pbase + c] = 0u;
    }
  }
  consumer_bar();
  if (ct < D) {
    // chunk order, then this (last) chunk: the same result whatever the timing
    float m2 = kNegBig, l2 = 0.f, a2 = 0.f;
    for (int c = 0; c <= active - 1; ++c) {
      float mc, lc, ac;
      if (c < active - 1) {
        mc = __ldcg(p.part_ml + (pbase + c) * 2);
        lc = __ldcg(p.part_ml + (pbase + c) * 2 + 1);
        ac = __ldcg(p.part_acc + (pbase + c) * D + ct);
      } else {
        mc = mm;
        lc = ll;
        ac = aa;
      }
      const float mn = fmaxf(m2, mc);
      const float w0 = exp2f(m2 - mn), w1 = exp2f(mc - mn);
      l2 = l2 * w0 + lc * w1;
      a2 = a2 * w0 + ac * w1;
      m2 = mn;
    }
    p.out[(size_t)bh * D + ct] = __float2half_rn(l2 > 0.f ? a2 / l2 : 0.f);
  }
  if (p.q_out) {
    consumer_bar();  // out[b, h] written by every thread before the count
    if (ct == 0) s.last_row = (atomic_add_acq_rel(p.cnt_row + b, 1) + 1 == p.H);
    consumer_bar();
    if (s.last_row) {
      // per-token quantisation of the attention row of b (as npl_quant_rows)
      const int n = p.H * D;
      const __half* row = p.out + (size_t)b * n;
      float amax = 0.f;
      for (int i = ct * 8; i < n; i += kAttnConsumers * 8) {
        float v[8];
        unpack8(__ldcg(reinterpret_cast<const uint4*>(row + i)), v);
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[j]));
      }
      amax = warp_max(amax);
      if ((ct & 31) == 0) s.red[ct >> 5] = amax;
      consumer_bar();
      amax = fmaxf(fmaxf(s.red[0], s.red[1]), fmaxf(s.red[2], s.red[3]));
      const float sc = scale_from_absmax(amax);
      const float rsc = quant_recip(sc);
      int8_t* qrow = p.q_out + (size_t)b * n;
      for (int i = ct * 8; i < n; i += kAttnConsumers * 8) {
        float v[8];
        unpack8(__ldcg(reinterpret_cast<const uint4*>(row + i)), v);
        uint2 u;
        uint32_t* w = reinterpret_cast<uint32_t*>(&u);
        w[0] = w[1] = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j / 4] |= (uint32_t)(quantize_one(v[j], sc, rsc) & 0xff) << (8 * (j % 4));
        *reinterpret_cast<uint2*>(qrow + i) = u;
      }
      if (ct == 0) {
        p.q_scale[b] = sc;
        p.cnt_row[b] = 0;
      }
    }
  }
  consumer_bar();  // stream state in shared memory is free for the next item
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads, kAttnCtasPerSm)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                       const AttnArgs p) {
  extern __shared__ unsigned char smem_raw[];
  AttnSmem<D>& s = *reinterpret_cast<AttnSmem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  constexpr int LPT = D / 8;  // lanes per token: 16 B of the head vector each
  constexpr int S = AttnSmem<D>::kStreams;
  constexpr int kPerStream = kAttnTok / S;
  constexpr int kU = kPerStream < 4 ? kPerStream : 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmap_k);
    prefetch_tensormap(&tmap_v);
    for (int i = 0; i < kAttnStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kAttnConsumers / 32);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const int bh_count = p.B * p.H;
      const int groups = p.H / p.Hkv;
      const uint32_t piece_bytes = (uint32_t)p.box_tok * D * sizeof(__half);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      // the first item of each CTA is blockIdx.x; the following ones come
      // from the work counter (which counts items beyond the first grid.x)
      int next = (int)blockIdx.x;
      while (ok) {
        const int item = next;
        if (item >= p.n_items) break;
        next = (int)gridDim.x + atomicAdd(p.work, 1);
        const int chunk = item / bh_count, bh = item % bh_count;
        const int b = bh / p.H, h = bh % p.H, kvh = h / groups;
        const int ctx = attn_ctx(p, b);
        const int t0 = chunk * kAttnChunk;
        if (t0 >= ctx && chunk > 0) continue;  // past the context: nothing to do
        const int t_end = min(ctx, t0 + kAttnChunk);
        const int n_st = max(1, (t_end - t0 + kAttnTok - 1) / kAttnTok);
        const int32_t* table = p.bt + (size_t)b * p.bt_stride;
        for (int st = 0; st < n_st && ok; ++st) {
          const int tok0 = t0 + st * kAttnTok;
          const int valid = max(0, min(kAttnTok, t_end - tok0));
          const int n_pieces = (valid + p.box_tok - 1) / p.box_tok;
          // block-table rows of the stage's pieces, read before waiting for a
          // free slot so their latency overlaps the wait
          int rows[kAttnTok / 8];
          int n_ok = 0;
#pragma unroll
          for (int i = 0; i < kAttnTok / 8; ++i) {
            rows[i] = -1;
            if (i < n_pieces) {
              const int tok = tok0 + i * p.box_tok;
              const int blk = table[tok / p.block_size];
              if (blk < 0 || blk >= p.num_blocks) {
                atomicCAS(p.status, 0, kDevBadIndex);
              } else {
                rows[i] = blk * p.block_size + tok % p.block_size;
                ++n_ok;
              }
            }
          }
          if (!mbar_wait(&s.empty[stage], phase ^ 1, p.status, NPL_DEV_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          s.meta[stage] = make_int4(item, st, valid, st == n_st - 1);
          const uint32_t q_bytes = st == 0 ? (uint32_t)D * sizeof(__half) : 0u;
          mbar_arrive_expect_tx(&s.full[stage], 2u * piece_bytes * (uint32_t)n_ok + q_bytes);
          if (st == 0) bulk_load(s.q[stage], p.q + (size_t)bh * D, q_bytes, &s.full[stage]);
#pragma unroll
          for (int i = 0; i < kAttnTok / 8; ++i) {
            if (rows[i] < 0) continue;
            tma_load_3d(s.k[stage] + i * p.box_tok * D, &tmap_k, 0, kvh, rows[i], &s.full[stage], pol);
            tma_load_3d(s.v[stage] + i * p.box_tok * D, &tmap_v, 0, kvh, rows[i], &s.full[stage], pol);
          }
          if (++stage == kAttnStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (ok && mbar_wait(&s.empty[stage], phase ^ 1, p.status, NPL_DEV_TIMEOUT_TMA)) {
        s.meta[stage] = make_int4(-1, 0, 0, 0);
        mbar_arrive(&s.full[stage]);
        // the last CTA to run out of work resets the work counters
        if (atomicAdd(p.work + 1, 1) + 1 == (int)gridDim.x) {
          atomicExch(p.work, 0);
          atomicExch(p.work + 1, 0);
        }
      }
    }
  } else {
    // --------------------------------------------------------- consumers
    const int ct = threadIdx.x - 32;
    const int stream = ct / LPT, sl = ct % LPT;
    const unsigned gmask = LPT == 32 ? 0xffffffffu : (((1u << LPT) - 1) << ((ct & 31) & ~(LPT - 1)));
    const float qscale = p.scale * 1.4426950408889634f;  // scores in log2 units
    float qv[8], acc[8];
    float m = kNegBig, l = 0.f;
    int stage = 0;
    uint32_t phase = 0;
    while (true) {
      if (!mbar_wait(&s.full[stage], phase, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) break;
      const volatile int* mv = reinterpret_cast<volatile int*>(&s.meta[stage]);
      const int4 meta = make_int4(mv[0], mv[1], mv[2], mv[3]);
      if (meta.x < 0) break;
      const int bh_count = p.B * p.H;
      const int chunk = meta.x / bh_count, bh = meta.x % bh_count;
      const int b = bh / p.H, h = bh % p.H;
      if (meta.y == 0) {
        unpack8(*reinterpret_cast<const uint4*>(s.q[stage] + sl * 8), qv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          qv[i] *= qscale;
          acc[i] = 0.f;
        }
        m = kNegBig;
        l = 0.f;
      }
      const __half* ks = s.k[stage];
      const __half* vs = s.v[stage];
#pragma unroll
      for (int j0 = 0; j0 < kPerStream; j0 += kU) {
        float sc[kU];
        float mnew = m;
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int t = stream + (j0 + u) * S;
          float kv[8];
          unpack8(*reinterpret_cast<const uint4*>(ks + t * D + sl * 8), kv);
          float d = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) d = fmaf(qv[i], kv[i], d);
#pragma unroll
          for (int o = LPT / 2; o > 0; o >>= 1) d += __shfl_xor_sync(gmask, d, o);
          sc[u] = t < meta.z ? d : -INFINITY;
          mnew = fmaxf(mnew, sc[u]);
        }
        const float alpha = exp2f(m - mnew);
        l *= alpha;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] *= alpha;
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int t = stream + (j0 + u) * S;
          if (t < meta.z) {
            const float pu = exp2f(sc[u] - mnew);
            l += pu;
            float vv[8];
            unpack8(*reinterpret_cast<const uint4*>(vs + t * D + sl * 8), vv);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fmaf(pu, vv[i], acc[i]);
          }
        }
        m = mnew;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[stage]);
      if (meta.w) attn_item_end<D>(p, s, ct, stream, sl, b, h, chunk, m, l, acc);
      if (++stage == kAttnStages) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
}

// fp16 cache [num_blocks * block_size][Hkv][D] as a 3-D tensor map; box =
// (D, 1 head, box_tok tokens).
int make_cache_map(CUtensorMap* map, const void* base, int num_blocks, int block_size, int Hkv, int D, int box_tok) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return fail(NPL_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)Hkv, (cuuint64_t)num_blocks * block_size};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)Hkv * D * 2};
  const cuuint32_t box[3] = {(cuuint32_t)D, 1, (cuuint32_t)box_tok};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NPL_ERR_ARG, "cuTensorMapEncodeTiled (KV cache) failed (%d)", (int)r);
  return NPL_OK;
}

// Workspace. The words that must be zero when a call starts sit at fixed
// offsets, so that calls of any shape can share one workspace: the work
// counters, one counter per sequence and one flag per (sequence, head,
// chunk); every call leaves them zero. The partials follow; their layout
// depends on the shape and they are always written before they are read.
constexpr size_t kAttnMaxParts = size_t(1) << 18;  // (sequence, head, chunk) per call

struct AttnLayout {
  size_t work, cnt_row, flags, ml, acc, total;
};

AttnLayout attn_layout(int B, int H, int D, int max_blocks, int block_size) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t n_chunks = std::max<size_t>(1, ((size_t)max_blocks * block_size + kAttnChunk - 1) / kAttnChunk);
  const size_t parts = (size_t)B * H * n_chunks;
  AttnLayout l;
  l.work = 0;
  l.cnt_row = 256;
  l.flags = l.cnt_row + al((size_t)kAttnMaxBatch * sizeof(int32_t));
  l.ml = l.flags + al(kAttnMaxParts * sizeof(uint32_t));
  l.acc = l.ml + al(parts * 2 * sizeof(float));
  l.total = l.acc + al(parts * D * sizeof(float));
  return l;
}

}  // namespace
}  // namespace npl

using namespace npl;

extern "C" int npl_store_kv(const void* key, const void* value, int ld_tok, int T, int Hkv, int D,
                            const int32_t* slot_mapping, void* k_cache, void* v_cache, int num_blocks,
                            int block_size, void* stream) {
  if (int rc = check_device()) return rc;
  if (!key || !value || !slot_mapping || !k_cache || !v_cache) return fail(NPL_ERR_ARG, "npl_store_kv: null pointer");
  if (T < 0 || Hkv <= 0 || D <= 0 || (Hkv * D) % 8 || ld_tok < Hkv * D || ld_tok % 8 || num_blocks <= 0 ||
      block_size <= 0)
    return fail(NPL_ERR_ARG, "npl_store_kv: bad shape");
  for (const void* p : std::initializer_list<const void*>{key, value, k_cache, v_cache})
    if (!aligned16(p)) return fail(NPL_ERR_ARG, "npl_store_kv: pointers must be 16-byte aligned");
  if (T == 0) return NPL_OK;
  return launch_pdl("npl_store_kv", store_kv_kernel, dim3(T), dim3(128), 0, static_cast<cudaStream_t>(stream),
                    static_cast<const __half*>(key), static_cast<const __half*>(value), ld_tok, Hkv * D,
                    slot_mapping, static_cast<__half*>(k_cache), static_cast<__half*>(v_cache),
                    (long long)num_blocks * block_size, device_status_ptr());
}

extern "C" int npl_rope_store_kv(const void* qkv, int ld_qkv, int T, int H, int Hkv, int D, const void* cos_table,
                                 const void* sin_table, int max_position, const int64_t* positions,
                                 const int32_t* slot_mapping, void* q_out, void* k_cache, void* v_cache,
                                 int num_blocks, int block_size, void* stream) {
  if (int rc = check_device()) return rc;
  if (!qkv || !cos_table || !sin_table || !positions || !slot_mapping || !q_out || !k_cache || !v_cache)
    return fail(NPL_ERR_ARG, "npl_rope_store_kv: null pointer");
  if (T < 0 || H <= 0 || Hkv <= 0 || H % Hkv || D <= 0 || D % 2 || D > 2048 || ld_qkv < (H + 2 * Hkv) * D ||
      max_position <= 0 || num_blocks <= 0 || block_size <= 0)
    return fail(NPL_ERR_ARG, "npl_rope_store_kv: bad shape");
  if (T == 0) return NPL_OK;
  // decode batches: one head per CTA; larger batches: every head of a token
  const int all_heads = H + 2 * Hkv;
  const int hpc = T <= 64 ? 1 : all_heads;
  const int threads = T <= 64 ? D / 2 : std::min(512, ((all_heads * D / 2 + 31) / 32) * 32);
  return launch_pdl("npl_rope_store_kv", rope_store_kernel, dim3(T, (all_heads + hpc - 1) / hpc), dim3(threads), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __half*>(qkv), ld_qkv, H, Hkv, D,
                    static_cast<const __half*>(cos_table), static_cast<const __half*>(sin_table), max_position,
                    positions, slot_mapping, static_cast<__half*>(q_out), static_cast<__half*>(k_cache),
                    static_cast<__half*>(v_cache), (long long)num_blocks * block_size, hpc, device_status_ptr());
}

extern "C" size_t npl_decode_attention_workspace_bytes(int B, int H, int D, int max_blocks, int block_size) {
  if (B <= 0 || H <= 0 || D <= 0 || max_blocks <= 0 || block_size <= 0) return 0;
  return attn_layout(B, H, D, max_blocks, block_size).total;
}

extern "C" int npl_paged_decode_attention(const void* q, int B, int H, int Hkv, int D, const void* k_cache,
                                          const void* v_cache, int num_blocks, int block_size,
                                          const int32_t* block_tables, int bt_stride, int max_blocks,
                                          const int32_t* context_lens, float scale, void* out, int8_t* q_out,
                                          float* q_scale, void* workspace, size_t workspace_bytes, void* stream) {
  if (int rc = check_device()) return rc;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out)
    return fail(NPL_ERR_ARG, "npl_paged_decode_attention: null pointer");
  if ((q_out == nullptr) != (q_scale == nullptr))
    return fail(NPL_ERR_ARG, "npl_paged_decode_attention: q_out and q_scale go together");
  if (B < 0 || H <= 0 || Hkv <= 0 || H % Hkv || num_blocks <= 0 || block_size <= 0 || max_blocks <= 0 ||
      bt_stride < max_blocks)
    return fail(NPL_ERR_ARG, "npl_paged_decode_attention: bad shape");
  if (D != 128 && D != 64) return fail(NPL_ERR_UNSUPPORTED, "npl_paged_decode_attention: head_dim %d (64 or 128)", D);
  if (block_size < 8 || (block_size % kAttnTok && kAttnTok % block_size))
    return fail(NPL_ERR_UNSUPPORTED,
                "npl_paged_decode_attention: block_size %d (a multiple of 64, or 8, 16 or 32)", block_size);
  for (const void* p : std::initializer_list<const void*>{q, k_cache, v_cache, out, (const void*)q_out})
    if (p && !aligned16(p)) return fail(NPL_ERR_ARG, "npl_paged_decode_attention: pointers must be 16-byte aligned");
  if (B == 0) return NPL_OK;
  if (B > kAttnMaxBatch)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_decode_attention: at most %d sequences per call", kAttnMaxBatch);
  if ((size_t)B * H * std::max(1, (max_blocks * block_size + kAttnChunk - 1) / kAttnChunk) > kAttnMaxParts)
    return fail(NPL_ERR_UNSUPPORTED, "npl_paged_decode_attention: more than %zu (sequence, head, %d-token chunk)",
                kAttnMaxParts, kAttnChunk);
  const AttnLayout lay = attn_layout(B, H, D, max_blocks, block_size);
  if (!workspace || workspace_bytes < lay.total || !aligned16(workspace))
    return fail(NPL_ERR_ARG, "npl_paged_decode_attention: workspace of %zu bytes required", lay.total);
  const int box_tok = std::min(kAttnTok, block_size);
  CUtensorMap tk, tv;
  if (int rc = make_cache_map(&tk, k_cache, num_blocks, block_size, Hkv, D, box_tok)) return rc;
  if (int rc = make_cache_map(&tv, v_cache, num_blocks, block_size, Hkv, D, box_tok)) return rc;
  char* ws = static_cast<char*>(workspace);
  AttnArgs p{};
  p.q = static_cast<const __half*>(q);
  p.B = B;
  p.H = H;
  p.Hkv = Hkv;
  p.num_blocks = num_blocks;
  p.block_size = block_size;
  p.box_tok = box_tok;
  p.bt = block_tables;
  p.bt_stride = bt_stride;
  p.max_blocks = max_blocks;
  p.ctx_lens = context_lens;
  p.scale = scale;
  p.n_chunks = std::max(1, (max_blocks * block_size + kAttnChunk - 1) / kAttnChunk);
  p.n_items = p.n_chunks * B * H;
  p.out = static_cast<__half*>(out);
  p.q_out = q_out;
  p.q_scale = q_scale;
  p.part_ml = reinterpret_cast<float*>(ws + lay.ml);
  p.part_acc = reinterpret_cast<float*>(ws + lay.acc);
  p.flags = reinterpret_cast<uint32_t*>(ws + lay.flags);
  p.cnt_row = reinterpret_cast<int32_t*>(ws + lay.cnt_row);
  p.work = reinterpret_cast<int32_t*>(ws + lay.work);
  p.status = device_status_ptr();
  const int sms = num_sms();
  const int grid = std::min(kAttnCtasPerSm * (sms > 0 ? sms : 148), p.n_items);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128) {
    const int smem = (int)sizeof(AttnSmem<128>) + 128;
    if (cudaFuncSetAttribute(decode_attn_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return launch_status("npl_paged_decode_attention: smem attribute");
    return launch_pdl("npl_paged_decode_attention", decode_attn_kernel<128>, dim3(grid), dim3(kAttnThreads),
                      (size_t)smem, st, tk, tv, p);
  }
  const int smem = (int)sizeof(AttnSmem<64>) + 128;
  if (cudaFuncSetAttribute(decode_attn_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return launch_status("npl_paged_decode_attention: smem attribute");
  return launch_pdl("npl_paged_decode_attention", decode_attn_kernel<64>, dim3(grid), dim3(kAttnThreads),
                    (size_t)smem, st, tk, tv, p);
}
