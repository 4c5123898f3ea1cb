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

// The same with 16-byte accesses: one thread per (token, head, 8 pair
// columns d .. d + 7 of the head's first half), so it moves 8 pairs per load
// of x1, x2, cos and sin. Used when D % 16 == 0 and every row is 16-byte
// aligned; same arithmetic per element as rope_store_kernel.
__device__ __forceinline__ void h8_load(const __half* p, float (&v)[8]) {
  const uint4 x = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__global__ void __launch_bounds__(256) rope_store_vec_kernel(const __half* __restrict__ qkv, int ld_qkv, int H,
                                                             int Hkv, int D, const __half* __restrict__ cos_t,
                                                             const __half* __restrict__ sin_t, int max_position,
                                                             const int64_t* __restrict__ positions,
                                                             const int32_t* __restrict__ slots,
                                                             __half* __restrict__ q_out, __half* __restrict__ kc,
                                                             __half* __restrict__ vc, long long num_slots,
                                                             long long items, int* status) {
  pdl_wait();
  pdl_trigger();
  const long long it = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (it >= items) return;
  const int half_d = D / 2, chunks = half_d / 8, all_heads = H + 2 * Hkv;
  const int d = (int)(it % chunks) * 8;
  const int head = (int)((it / chunks) % all_heads);
  const long long t = it / chunks / all_heads;
  const long long pos = positions[t];
  const long long slot = slots[t];
  const bool pos_ok = pos >= 0 && pos < max_position;
  const bool slot_ok = slot >= 0 && slot < num_slots;
  if (head == 0 && d == 0 && (!pos_ok || slot >= num_slots)) flag_bad_index(status);
  const __half* x = qkv + t * ld_qkv + (size_t)head * D;
  if (head >= H + Hkv) {  // v
    if (slot_ok) {
      __half* vd = vc + (slot * Hkv + (head - H - Hkv)) * D;
      *reinterpret_cast<uint4*>(vd + d) = *reinterpret_cast<const uint4*>(x + d);
      *reinterpret_cast<uint4*>(vd + d + half_d) = *reinterpret_cast<const uint4*>(x + d + half_d);
    }
    return;
  }
  if (!pos_ok) return;
  __half* dst;
  if (head < H) {
    dst = q_out + ((size_t)t * H + head) * D;
  } else {
    if (!slot_ok) return;
    dst = kc + (slot * Hkv + (head - H)) * D;
  }
  float x1[8], x2[8], c1[8], c2[8], s1[8], s2[8];
  h8_load(x + d, x1);
  h8_load(x + d + half_d, x2);
  h8_load(cos_t + pos * D + d, c1);
  h8_load(cos_t + pos * D + d + half_d, c2);
  h8_load(sin_t + pos * D + d, s1);
  h8_load(sin_t + pos * D + d + half_d, s2);
  uint4 o1, o2;
  __half* h1 = reinterpret_cast<__half*>(&o1);
  __half* h2 = reinterpret_cast<__half*>(&o2);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a1 = __half2float(__float2half_rn(__fmul_rn(x1[i], c1[i])));
    const float b1 = __half2float(__float2half_rn(__fmul_rn(-x2[i], s1[i])));
    const float a2 = __half2float(__float2half_rn(__fmul_rn(x2[i], c2[i])));
    const float b2 = __half2float(__float2half_rn(__fmul_rn(x1[i], s2[i])));
    h1[i] = __float2half_rn(__fadd_rn(a1, b1));
    h2[i] = __float2half_rn(__fadd_rn(a2, b2));
  }
  *reinterpret_cast<uint4*>(dst + d) = o1;
  *reinterpret_cast<uint4*>(dst + d + half_d) = o2;
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

// The same with an L2 cache-eviction policy (createpolicy).
__device__ __forceinline__ void bulk_load_pol(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
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

// --------------------------------------- paged decode attention, row streams
// The kernel for head_dim 128 (the 7B geometry and any H multiple of 4 up to
// 64). One CTA per SM; a work unit is (64-token chunk of a sequence's
// context) x EVERY head, so the CTA streams whole cache rows: each token's K
// (and V) row of all kv heads is contiguous (Hkv x 256 bytes; 8 KB at the 7B
// geometry), and the tokens of a chunk inside one cache block are contiguous
// too, so every copy is one 1-D bulk copy of several KB. Units are numbered
// from a prefix sum of the sequences' unit counts (built in shared memory by
// every CTA, so no number is an empty unit): first every unit but the last of
// each sequence, sequence by sequence, then the last (partly filled) unit of
// every sequence, so the light units come last. Each CTA starts with unit
// blockIdx.x and takes the next ones from a work counter, which keeps the
// CTAs balanced when the contexts are ragged.
//
//   warp 0         producer: for each unit, ring stages of tok_stage tokens
//                  (K rows then V rows, ~32 KB each) by cp.async.bulk
//   warps 1..      consumers: H/2 warps of 2 q-heads (16 lanes per head, 8
//                  dims per lane) for H <= 32, else H/4 warps of 4 q-heads
//                  (8 lanes, 16 dims); a quarter-warp always reads 128
//                  contiguous bytes (no bank conflicts); one online softmax
//                  per head over the unit. q . k runs as fp16 x fp16
//                  products accumulated in fp32 by mixed-precision FMA (the
//                  fp16 operands need no conversion); p * v in fp32.
//
// Every unit ends in a partial (max, sum, acc[D]) per head. A sequence with
// one unit (context <= 64) is finished right there; otherwise its units write
// their partials and the unit that completes the sequence (a per-sequence
// counter) merges all of them in chunk order and writes out[b]. The split of
// a sequence depends only on its own context length, never on the rest of the
// batch, so a sequence's result is the same in any batch. With q_out, the
// CTA that finishes a sequence also quantises its attention row per token
// (as npl_quant_rows), the O projection's input.
constexpr int kRowUnit = 64;
constexpr int kRowMaxWarps = 16;  // consumer warps: H <= 64
constexpr int kRowStageTarget = 32 * 1024;
constexpr int kRowSmemBudget = 200 * 1024;

struct RowArgs {
  const __half* q;
  int B, H, Hkv;
  const unsigned char* kc;  // [num_blocks * block_size] rows of row_bytes
  const unsigned char* vc;
  int num_blocks, block_size;
  const int32_t* bt;
  int bt_stride, max_blocks;
  const int32_t* ctx_lens;
  float scale;
  int n_chunks;   // 64-token units per sequence at most
  int tok_stage;  // tokens per ring stage (divides 64)
  int n_stages;
  int row_bytes;  // Hkv * 128 * 2
  __half* out;
  int8_t* q_out;
  float* q_scale;
  float* part_ml;   // [B][n_chunks][H][2]
  float* part_acc;  // [B][n_chunks][H][128]
  int32_t* cnt;     // [B]: units finished (reset by the unit that merges)
  int32_t* work;    // [2]: units handed out beyond the first grid.x; CTAs done (reset by the last CTA)
  int* status;
};

__device__ __forceinline__ void rows_bar(int nthreads) {
  asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

__device__ __forceinline__ int rows_ctx(const RowArgs& p, int b) {
  return min(max(0, p.ctx_lens[b]), p.max_blocks * p.block_size);
}


// An fp16 pair as two fp32 values.
__device__ __forceinline__ float2 h2f2(uint32_t x) {
  __half2 h = *reinterpret_cast<__half2*>(&x);
  return __half22float2(h);
}
// d_lo += x.lo * y.lo and d_hi += x.hi * y.hi for fp16 pairs x, y, with the
// fp16 x fp16 products (exact in fp32) accumulated in fp32 (mixed-precision
// FMA: no conversion of the fp16 operands to fp32 first).
__device__ __forceinline__ void fma2_f32_f16(float& d_lo, float& d_hi, uint32_t x, uint32_t y) {
  asm("{.reg .f16 xl, xh, yl, yh;\n\t"
      "mov.b32 {xl, xh}, %2;\n\t"
      "mov.b32 {yl, yh}, %3;\n\t"
      "fma.rn.f32.f16 %0, xl, yl, %0;\n\t"
      "fma.rn.f32.f16 %1, xh, yh, %1;}"
      : "+f"(d_lo), "+f"(d_hi)
      : "r"(x), "r"(y));
}


// Lane layout of the consumers, for DPL (dims per lane) 8 or 16: a head's
// 128 dims are spread over LPH = 128 / DPL lanes, each holding DPL / 8
// 16-byte chunks (chunk c at byte c * 128 + 16 j of the head, j < LPH), so a
// quarter-warp always reads 128 contiguous bytes; a warp covers HPW = 32 / LPH
// q-heads.
template <int DPL>
struct RowLanes {
  static constexpr int LPH = 128 / DPL;
  static constexpr int HPW = 32 / LPH;
  static constexpr int CH = DPL / 8;  // 16-byte chunks per lane
};

// The lane's chunks of a cache row (or q row), as DPL / 2 fp16 pairs.
template <int DPL>
__device__ __forceinline__ void load_pairs(const unsigned char* row, int off, uint32_t (&v)[DPL / 2]) {
#pragma unroll
  for (int c = 0; c < DPL / 8; ++c) {
    const uint4 a = *reinterpret_cast<const uint4*>(row + off + c * 128);
    v[4 * c] = a.x;
    v[4 * c + 1] = a.y;
    v[4 * c + 2] = a.z;
    v[4 * c + 3] = a.w;
  }
}

// out[b, hq] (and the int8 row of b) from a finished (sum, acc); every
// consumer thread of the CTA calls it together.
template <int DPL>
__device__ void rows_finish(const RowArgs& p, float* red, int nthreads, int cw, int lane, int b, int hq, int j,
                            float l, const float (&acc)[DPL]) {
  __half o[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) o[i] = __float2half_rn(l > 0.f ? acc[i] / l : 0.f);
  __half* orow = p.out + ((size_t)b * p.H + hq) * 128;
#pragma unroll
  for (int c = 0; c < DPL / 8; ++c)
    *reinterpret_cast<uint4*>(orow + 64 * c + 8 * j) = *reinterpret_cast<const uint4*>(&o[8 * c]);
  if (!p.q_out) return;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < DPL; ++i) amax = fmaxf(amax, fabsf(__half2float(o[i])));
  amax = warp_max(amax);
  if (lane == 0) red[cw] = amax;
  rows_bar(nthreads);
  amax = 0.f;
  for (int i = 0; i < nthreads / 32; ++i) amax = fmaxf(amax, red[i]);
  const float sc = scale_from_absmax(amax);
  const float rsc = quant_recip(sc);
  int8_t* qrow = p.q_out + ((size_t)b * p.H + hq) * 128;
#pragma unroll
  for (int c = 0; c < DPL / 8; ++c) {
    uint2 u;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
    w[0] = w[1] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      w[i / 4] |= (uint32_t)(quantize_one(__half2float(o[8 * c + i]), sc, rsc) & 0xff) << (8 * (i % 4));
    *reinterpret_cast<uint2*>(qrow + 64 * c + 8 * j) = u;
  }
  if (cw == 0 && lane == 0) p.q_scale[b] = sc;
  rows_bar(nthreads);  // red[] is free again
}

// Merges the partials of sequence b (every unit of it has written its
// partial) in chunk order and writes out[b]; every consumer thread of the CTA
// calls it together.
template <int DPL>
__device__ void rows_merge(const RowArgs& p, float* red, int nthreads, int cw, int lane, int b, int hq, int j) {
  using LN = RowLanes<DPL>;
  const int n_b = max(1, (rows_ctx(p, b) + kRowUnit - 1) / kRowUnit);
  float mm = kNegBig, ll = 0.f, aa[DPL];
#pragma unroll
  for (int i = 0; i < DPL; ++i) aa[i] = 0.f;
  for (int cidx = 0; cidx < n_b; ++cidx) {
    const size_t pc = ((size_t)b * p.n_chunks + cidx) * p.H + hq;
    const float2 ml = __ldcg(reinterpret_cast<const float2*>(p.part_ml) + pc);
    const float4* src = reinterpret_cast<const float4*>(p.part_acc + pc * 128);
    float ac[DPL];
#pragma unroll
    for (int c = 0; c < LN::CH; ++c) {
      const float4 x0 = __ldcg(src + 16 * c + 2 * j), x1 = __ldcg(src + 16 * c + 2 * j + 1);
      ac[8 * c] = x0.x; ac[8 * c + 1] = x0.y; ac[8 * c + 2] = x0.z; ac[8 * c + 3] = x0.w;
      ac[8 * c + 4] = x1.x; ac[8 * c + 5] = x1.y; ac[8 * c + 6] = x1.z; ac[8 * c + 7] = x1.w;
    }
    const float mn = fmaxf(mm, ml.x);
    const float w0 = exp2f(mm - mn), w1 = exp2f(ml.x - mn);
    ll = ll * w0 + ml.y * w1;
#pragma unroll
    for (int i = 0; i < DPL; ++i) aa[i] = aa[i] * w0 + ac[i] * w1;
    mm = mn;
  }
  if (cw == 0 && lane == 0) p.cnt[b] = 0;  // no other unit of this launch counts b again
  rows_finish<DPL>(p, red, nthreads, cw, lane, b, hq, j, ll, aa);
}

template <int DPL>
__global__ void __launch_bounds__(32 * (kRowMaxWarps + 1), 1) decode_attn_rows_kernel(const RowArgs p) {
  using LN = RowLanes<DPL>;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                                         ~uintptr_t(127));
  const int nw = (int)(blockDim.x >> 5) - 1;  // consumer warps
  const int nthreads = nw * 32;
  const size_t stage_bytes = (size_t)p.tok_stage * p.row_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * (size_t)p.n_stages * stage_bytes);
  uint64_t* empty = full + p.n_stages;
  int4* meta = reinterpret_cast<int4*>(empty + p.n_stages);
  float* red = reinterpret_cast<float*>(meta + p.n_stages);
  int* merge_slot = reinterpret_cast<int*>(red + kRowMaxWarps);  // [2]
  int* unit_start = merge_slot + 4;                                // [B + 1]: first unit of each sequence
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.n_stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], nw);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    // unit_start[b] = units of the sequences before b (a warp scan per 32 sequences)
    int run = 0;
    for (int b0 = 0; b0 < p.B; b0 += 32) {
      const int b = b0 + lane;
      int x = b < p.B ? max(1, (rows_ctx(p, b) + kRowUnit - 1) / kRowUnit) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (b < p.B) unit_start[b + 1] = run + x;
      run += __shfl_sync(0xffffffffu, x, 31);
    }
    __syncwarp();  // the other lanes' entries before lane 0 reads them
    if (lane != 0) return;
    unit_start[0] = 0;
    const int n_units = run;
    const uint64_t pol = policy_evict_first();
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used = 0, parity = 0;  // per ring slot: issued at least once; parity of its last phase
    bool ok = true;
    // the first unit of each CTA is blockIdx.x; the following ones come from
    // the work counter (which counts units beyond the first grid.x), when
    // there are more units than CTAs
    const bool dynamic = n_units > (int)gridDim.x;
    int next = (int)blockIdx.x;
    while (ok) {
      const int u = next;
      if (u >= n_units) break;
      next = dynamic ? (int)gridDim.x + atomicAdd(p.work, 1) : n_units;
      // units [0, n_units - B): the non-last units, sequence b's starting at
      // unit_start[b] - b; units [n_units - B, n_units): the last units
      const int n_inner = n_units - p.B;
      int b, chunk;
      if (u < n_inner) {
        b = 0;  // the last b with unit_start[b] - b <= u
        for (int hi = p.B - 1; b < hi;) {
          const int mid = (b + hi + 1) >> 1;
          if (unit_start[mid] - mid <= u) b = mid;
          else hi = mid - 1;
        }
        chunk = u - (unit_start[b] - b);
      } else {
        b = u - n_inner;
        chunk = unit_start[b + 1] - unit_start[b] - 1;
      }
      const int ctx = rows_ctx(p, b);
      const int t0 = chunk * kRowUnit, t_end = min(ctx, t0 + kRowUnit);
      const int n_st = max(1, (t_end - t0 + p.tok_stage - 1) / p.tok_stage);
      const int32_t* table = p.bt + (size_t)b * p.bt_stride;
      for (int st = 0; st < n_st; ++st) {
        const int tok0 = t0 + st * p.tok_stage;
        int valid = max(0, min(p.tok_stage, t_end - tok0));
        // pieces: runs of the stage's tokens inside one cache block (at most
        // 64 / 8: block_size >= 8, tok_stage <= 64)
        const int piece = min(p.tok_stage, p.block_size);
        long long rows[kRowUnit / 8];
        int n_pieces = min((valid + piece - 1) / piece, kRowUnit / 8);
        for (int i = 0; i < n_pieces; ++i) {
          const int tok = tok0 + i * piece;
          const int blk = table[tok / p.block_size];
          if (blk < 0 || blk >= p.num_blocks) {
            atomicCAS(p.status, 0, kDevBadIndex);
            valid = 0;  // the stage is skipped (its tokens count as masked)
            n_pieces = 0;
            break;
          }
          rows[i] = (long long)blk * p.block_size + tok % p.block_size;
        }
        if (!mbar_wait(&empty[stage], phase ^ 1, p.status, NPL_DEV_TIMEOUT_TMA)) {
          ok = false;
          break;
        }
        meta[stage] = make_int4(chunk * p.B + b, st, valid, st == n_st - 1);
        used |= 1u << stage;
        parity = (parity & ~(1u << stage)) | (phase << stage);
        mbar_arrive_expect_tx(&full[stage], 2u * (uint32_t)valid * (uint32_t)p.row_bytes);
        unsigned char* kdst = smem + (size_t)(2 * stage) * stage_bytes;
        unsigned char* vdst = kdst + stage_bytes;
        for (int i = 0; i < n_pieces; ++i) {
          const int ntok = min(piece, valid - i * piece);
          const uint32_t bytes = (uint32_t)ntok * (uint32_t)p.row_bytes;
          const size_t src = (size_t)rows[i] * p.row_bytes;
          const size_t dst = (size_t)i * piece * p.row_bytes;
          bulk_load_pol(kdst + dst, p.kc + src, bytes, &full[stage], pol);
          bulk_load_pol(vdst + dst, p.vc + src, bytes, &full[stage], pol);
        }
        if (++stage == p.n_stages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    if (ok && mbar_wait(&empty[stage], phase ^ 1, p.status, NPL_DEV_TIMEOUT_TMA)) {
      meta[stage] = make_int4(-1, 0, 0, 0);
      used |= 1u << stage;
      parity = (parity & ~(1u << stage)) | (phase << stage);
      mbar_arrive(&full[stage]);
    }
    // every CTA counts itself done after its last take from the work counter;
    // the last one resets both words for the next launch
    if (dynamic && atomicAdd(p.work + 1, 1) + 1 == (int)gridDim.x) {
      atomicExch(p.work, 0);
      atomicExch(p.work + 1, 0);
    }
    // Copies land before the CTA exits: the last phase of every slot that was
    // issued has completed (at once, unless a wait above expired).
    for (int i = 0; i < p.n_stages; ++i)
      if (used >> i & 1) mbar_wait(&full[i], parity >> i & 1, p.status, NPL_DEV_TIMEOUT_TEARDOWN);
    return;
  }

  // ------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int hq = cw * LN::HPW + lane / LN::LPH;  // q-head of this lane
  const int j = lane % LN::LPH;                  // chunk c covers dims 64 c + 8 j .. + 8
  const int kvh = hq / (p.H / p.Hkv);
  const int koff = kvh * 256 + j * 16;  // byte offset of the lane's first chunk in a cache row
  const float qscale = p.scale * 1.4426950408889634f;  // scores in log2 units
  uint32_t qv[DPL / 2];  // the lane's query values, fp16 pairs (scaled after the dot)
  float acc[DPL];        // the same dims, in pair order
  float m = kNegBig, l = 0.f;
  int stage = 0;
  uint32_t phase = 0;
  // The count at the end of a unit is taken by thread 0 without waiting for
  // it; its outcome (this unit completes sequence pend_b) is published at the
  // next unit end, or after the last unit, through merge_slot[slot].
  int pend_b = -1, slot = 0;
  bool pend_last = false, done = false;
  while (true) {
    if (!mbar_wait(&full[stage], phase, p.status, NPL_DEV_TIMEOUT_EPILOGUE)) break;
    const volatile int* mv = reinterpret_cast<volatile int*>(&meta[stage]);
    const int4 mt = make_int4(mv[0], mv[1], mv[2], mv[3]);
    if (mt.x < 0) {
      done = true;
      break;
    }
    const int chunk = mt.x / p.B, b = mt.x % p.B;
    if (mt.y == 0) {
      const unsigned char* qrow = reinterpret_cast<const unsigned char*>(p.q + ((size_t)b * p.H + hq) * 128);
#pragma unroll
      for (int c = 0; c < LN::CH; ++c) {
        const uint4 a = __ldcg(reinterpret_cast<const uint4*>(qrow + c * 128 + j * 16));
        qv[4 * c] = a.x;
        qv[4 * c + 1] = a.y;
        qv[4 * c + 2] = a.z;
        qv[4 * c + 3] = a.w;
      }
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
      m = kNegBig;
      l = 0.f;
    }
    const unsigned char* ks = smem + (size_t)(2 * stage) * stage_bytes;
    const unsigned char* vs = ks + stage_bytes;
    for (int t0 = 0; t0 < mt.z; t0 += 4) {
      float sc[4];
      float mnew = m;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = min(t0 + u, mt.z - 1);
        uint32_t kv[DPL / 2];
        load_pairs<DPL>(ks + (size_t)t * p.row_bytes, koff, kv);
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;  // four chains of q . k over the lane's dims
#pragma unroll
        for (int i = 0; i < DPL / 2; i += 2) {
          fma2_f32_f16(d0, d1, qv[i], kv[i]);
          fma2_f32_f16(d2, d3, qv[i + 1], kv[i + 1]);
        }
        float d = (d0 + d1) + (d2 + d3);
#pragma unroll
        for (int o = LN::LPH / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        sc[u] = t0 + u < mt.z ? d * qscale : -INFINITY;
        mnew = fmaxf(mnew, sc[u]);
      }
      const float alpha = exp2f(m - mnew);
      l *= alpha;
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] *= alpha;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (t0 + u < mt.z) {
          const float pu = exp2f(sc[u] - mnew);
          l += pu;
          
          uint32_t vv[DPL / 2];
          load_pairs<DPL>(vs + (size_t)(t0 + u) * p.row_bytes, koff, vv);
#pragma unroll
          for (int i = 0; i < DPL / 2; ++i) {
            const float2 f = h2f2(vv[i]);
            acc[2 * i] = fmaf(pu, f.x, acc[2 * i]);
            acc[2 * i + 1] = fmaf(pu, f.y, acc[2 * i + 1]);
          }
        }
      }
      m = mnew;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == p.n_stages) {
      stage = 0;
      phase ^= 1;
    }
    if (!mt.w) continue;

    // ---- end of a unit
    const int n_b = max(1, (rows_ctx(p, b) + kRowUnit - 1) / kRowUnit);
    if (n_b == 1) {
      rows_finish<DPL>(p, red, nthreads, cw, lane, b, hq, j, l, acc);
      continue;
    }
    const size_t pi = ((size_t)b * p.n_chunks + chunk) * p.H + hq;
    if (j == 0) __stcg(reinterpret_cast<float2*>(p.part_ml) + pi, make_float2(m, l));
    float4* pa = reinterpret_cast<float4*>(p.part_acc + pi * 128);
#pragma unroll
    for (int c = 0; c < LN::CH; ++c) {
      __stcg(pa + 16 * c + 2 * j, make_float4(acc[8 * c], acc[8 * c + 1], acc[8 * c + 2], acc[8 * c + 3]));
      __stcg(pa + 16 * c + 2 * j + 1, make_float4(acc[8 * c + 4], acc[8 * c + 5], acc[8 * c + 6], acc[8 * c + 7]));
    }
    if (cw == 0 && lane == 0) merge_slot[slot] = pend_last ? pend_b : -1;
    rows_bar(nthreads);  // every partial write of the CTA before the count (cumulative release); the slot
    const int mb = merge_slot[slot];
    slot ^= 1;  // (two slots: thread 0 may write the next one before a slow thread has read this one)
    if (cw == 0 && lane == 0) {
      pend_b = b;
      pend_last = atomic_add_acq_rel(p.cnt + b, 1) + 1 == n_b;
    }
    if (mb >= 0) rows_merge<DPL>(p, red, nthreads, cw, lane, mb, hq, j);
  }
  if (!done) return;  // a bounded wait gave up (the status word says so)
  if (cw == 0 && lane == 0) merge_slot[slot] = pend_last ? pend_b : -1;
  rows_bar(nthreads);
  const int mb = merge_slot[slot];
  if (mb >= 0) rows_merge<DPL>(p, red, nthreads, cw, lane, mb, hq, j);
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

// The partials are sized for both kernels: (sequence, head, 256-token chunk)
// of decode_attn_kernel and (sequence, 64-token unit, head) of
// decode_attn_rows_kernel; the per-sequence counters are shared (both leave
// them zero).
AttnLayout attn_layout(int B, int H, int D, int max_blocks, int block_size) {
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t ctx = (size_t)max_blocks * block_size;
  const size_t n_chunks = std::max<size_t>(1, (ctx + kAttnChunk - 1) / kAttnChunk);
  const size_t n_units = std::max<size_t>(1, (ctx + kRowUnit - 1) / kRowUnit);
  const size_t parts = std::max((size_t)B * H * n_chunks, (size_t)B * H * n_units);
  AttnLayout l;
  l.work = 0;
  l.cnt_row = 256;
  l.flags = l.cnt_row + al((size_t)kAttnMaxBatch * sizeof(int32_t));
  l.ml = l.flags + al(kAttnMaxParts * sizeof(uint32_t));
  l.acc = l.ml + al(parts * 2 * sizeof(float));
  l.total = l.acc + al(parts * D * sizeof(float));
  return l;
}

// Ring configuration of decode_attn_rows_kernel for this geometry (0 stages:
// not supported, use decode_attn_kernel).
struct RowConfig {
  int tok_stage, n_stages, row_bytes, warps;
  size_t smem;
};

// Consumer layout: 8 dims per lane (2 q-heads per warp) while H / 2 warps fit,
// else 16 dims per lane (4 q-heads per warp).
RowConfig row_config(int H, int Hkv, int D, int block_size) {
  RowConfig c{0, 0, Hkv * D * 2, H % 2 == 0 && H / 2 <= kRowMaxWarps ? H / 2 : H / 4, 0};
  if (D != 128 || H % 4 || H / 4 > kRowMaxWarps || H % Hkv) return c;
  int t = kRowUnit;
  while (t > 1 && (size_t)t * c.row_bytes > kRowStageTarget) t /= 2;
  if (block_size % t && t % block_size) return c;
  const size_t stage = (size_t)t * c.row_bytes;
  const int n = (int)std::min<size_t>(4, kRowSmemBudget / (2 * stage));
  if (n < 2) return c;
  c.tok_stage = t;
  c.n_stages = n;
  c.smem = 128 + 2 * (size_t)n * stage + n * (2 * sizeof(uint64_t) + sizeof(int4)) + kRowMaxWarps * sizeof(float) + 16;
  return c;
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
  const int all_heads = H + 2 * Hkv;
  if (D % 16 == 0 && ld_qkv % 8 == 0 && aligned16(qkv) && aligned16(cos_table) && aligned16(sin_table) &&
      aligned16(q_out) && aligned16(k_cache) && aligned16(v_cache)) {
    const long long items = (long long)T * all_heads * (D / 16);
    return launch_pdl("npl_rope_store_kv", rope_store_vec_kernel, dim3((unsigned)((items + 255) / 256)), dim3(256),
                      0, static_cast<cudaStream_t>(stream), static_cast<const __half*>(qkv), ld_qkv, H, Hkv, D,
                      static_cast<const __half*>(cos_table), static_cast<const __half*>(sin_table), max_position,
                      positions, slot_mapping, static_cast<__half*>(q_out), static_cast<__half*>(k_cache),
                      static_cast<__half*>(v_cache), (long long)num_blocks * block_size, items,
                      device_status_ptr());
  }
  // decode batches: one head per CTA; larger batches: every head of a token
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
  const RowConfig rc = row_config(H, Hkv, D, block_size);
  if (rc.n_stages > 0) {
    char* ws = static_cast<char*>(workspace);
    RowArgs r{};
    r.q = static_cast<const __half*>(q);
    r.B = B;
    r.H = H;
    r.Hkv = Hkv;
    r.kc = static_cast<const unsigned char*>(k_cache);
    r.vc = static_cast<const unsigned char*>(v_cache);
    r.num_blocks = num_blocks;
    r.block_size = block_size;
    r.bt = block_tables;
    r.bt_stride = bt_stride;
    r.max_blocks = max_blocks;
    r.ctx_lens = context_lens;
    r.scale = scale;
    r.n_chunks = std::max(1, (max_blocks * block_size + kRowUnit - 1) / kRowUnit);
    r.tok_stage = rc.tok_stage;
    r.n_stages = rc.n_stages;
    r.row_bytes = rc.row_bytes;
    r.out = static_cast<__half*>(out);
    r.q_out = q_out;
    r.q_scale = q_scale;
    r.part_ml = reinterpret_cast<float*>(ws + lay.ml);
    r.part_acc = reinterpret_cast<float*>(ws + lay.acc);
    r.cnt = reinterpret_cast<int32_t*>(ws + lay.cnt_row);
    r.work = reinterpret_cast<int32_t*>(ws + lay.work);
    r.status = device_status_ptr();
    const int sms = num_sms();
    const long long units = (long long)r.n_chunks * B;
    const int grid = (int)std::min<long long>(sms > 0 ? sms : 148, units);
    auto kern = rc.warps * 2 == H ? decode_attn_rows_kernel<8> : decode_attn_rows_kernel<16>;
    const size_t smem = rc.smem + (size_t)(B + 1) * sizeof(int);  // + unit_start
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return launch_status("npl_paged_decode_attention: smem attribute");
    return launch_pdl("npl_paged_decode_attention", kern, dim3(grid), dim3(32 * (rc.warps + 1)), smem,
                      static_cast<cudaStream_t>(stream), r);
  }
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
