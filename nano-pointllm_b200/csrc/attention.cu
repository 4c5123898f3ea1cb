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

#include "npl_common.cuh"

namespace npl {
namespace {

constexpr int kDevBadIndex = 5;  // a slot, block or position outside its table

__device__ __forceinline__ void flag_bad_index(int* status) {
  if (status) atomicCAS(status, 0, kDevBadIndex);
}

// ------------------------------------------------------------ store_kvcache
__global__ void store_kv_kernel(const __half* __restrict__ key, const __half* __restrict__ value, int ld_tok,
                                int hkv_d, const int32_t* __restrict__ slots, __half* __restrict__ kc,
                                __half* __restrict__ vc, long long num_slots, int* status) {
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
// One CTA per token. Pair (d, d + D/2) of each q/k head:
//   out[d]       = fp16(fp16(x1 * cos[d])       + fp16(-x2 * sin[d]))
//   out[d + D/2] = fp16(fp16(x2 * cos[d + D/2]) + fp16( x1 * sin[d + D/2]))
// (HF apply_rotary_pos_emb with rotate_half(x) = cat(-x2, x1), each torch
// fp16 op rounded once).
__global__ void rope_store_kernel(const __half* __restrict__ qkv, int ld_qkv, int H, int Hkv, int D,
                                  const __half* __restrict__ cos_t, const __half* __restrict__ sin_t,
                                  int max_position, const int64_t* __restrict__ positions,
                                  const int32_t* __restrict__ slots, __half* __restrict__ q_out,
                                  __half* __restrict__ kc, __half* __restrict__ vc, long long num_slots,
                                  int* status) {
  const int t = blockIdx.x;
  const long long pos = positions[t];
  const long long slot = slots[t];
  const __half* row = qkv + (size_t)t * ld_qkv;
  const int half_d = D / 2;
  const bool pos_ok = pos >= 0 && pos < max_position;
  const bool slot_ok = slot >= 0 && slot < num_slots;
  if (threadIdx.x == 0 && (!pos_ok || slot >= num_slots)) flag_bad_index(status);
  if (!pos_ok) return;
  const __half* c = cos_t + pos * D;
  const __half* s = sin_t + pos * D;
  const int n_pairs = (H + Hkv) * half_d;
  for (int i = threadIdx.x; i < n_pairs; i += blockDim.x) {
    const int head = i / half_d, d = i - head * half_d;
    const float x1 = __half2float(row[head * D + d]);
    const float x2 = __half2float(row[head * D + d + half_d]);
    const float a1 = __half2float(__float2half_rn(__fmul_rn(x1, __half2float(c[d]))));
    const float b1 = __half2float(__float2half_rn(__fmul_rn(-x2, __half2float(s[d]))));
    const float a2 = __half2float(__float2half_rn(__fmul_rn(x2, __half2float(c[d + half_d]))));
    const float b2 = __half2float(__float2half_rn(__fmul_rn(x1, __half2float(s[d + half_d]))));
    const __half o1 = __float2half_rn(__fadd_rn(a1, b1));
    const __half o2 = __float2half_rn(__fadd_rn(a2, b2));
    if (head < H) {
      __half* qo = q_out + ((size_t)t * H + head) * D;
      qo[d] = o1;
      qo[d + half_d] = o2;
    } else if (slot_ok) {
      __half* kd = kc + (slot * Hkv + (head - H)) * D;
      kd[d] = o1;
      kd[d + half_d] = o2;
    }
  }
  if (slot_ok) {
    const __half* v = row + (H + Hkv) * D;
    __half* vd = vc + slot * Hkv * D;
    for (int i = threadIdx.x; i < Hkv * D; i += blockDim.x) vd[i] = v[i];
  }
}

// ------------------------------------------------- paged decode attention
// Grid (splits, H, B); CTA = 4 warps; each half-warp (D = 128: 16 lanes x 8
// dims) is a token stream with its own online-softmax state over the CTA's
// chunk of the context. Streams merge in shared memory; each CTA writes a
// partial (max, sum, acc[D]); the last CTA of (b, h) merges the splits and
// writes the fp16 output.
constexpr int kAttnThreads = 128;
constexpr int kUnroll = 4;
constexpr float kNegBig = -1.0e30f;

template <int D>
struct AttnCfg {
  static constexpr int kLanesPerTok = D / 8;               // 16 B per lane
  static constexpr int kStreams = kAttnThreads / kLanesPerTok;
};

__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
  const uint4 x = __ldcs(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads)
    decode_attn_kernel(const __half* __restrict__ q, int H, int Hkv, const __half* __restrict__ kc,
                       const __half* __restrict__ vc, int num_blocks, int block_size,
                       const int32_t* __restrict__ bt, int bt_stride, int max_blocks,
                       const int32_t* __restrict__ ctx_lens, float scale, int chunk, __half* __restrict__ out,
                       float* __restrict__ part_ml, float* __restrict__ part_acc, int32_t* __restrict__ counters,
                       int* status) {
  using C = AttnCfg<D>;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int n_splits = gridDim.x;
  // a context longer than the block table row is clamped (and flagged)
  const int ctx_raw = ctx_lens[b];
  const int ctx = min(max(0, ctx_raw), max_blocks * block_size);
  if (ctx != max(0, ctx_raw) && split == 0 && h == 0 && threadIdx.x == 0) flag_bad_index(status);
  const int active = max(1, (ctx + chunk - 1) / chunk);
  if (split >= active) return;
  const int kvh = h / (H / Hkv);
  const int tid = threadIdx.x;
  const int stream = tid / C::kLanesPerTok;
  const int sl = tid % C::kLanesPerTok;  // lane within the token stream
  const unsigned grp_mask = C::kLanesPerTok == 32 ? 0xffffffffu
                                                  : (((1u << C::kLanesPerTok) - 1) << ((tid & 31) & ~(C::kLanesPerTok - 1)));

  float qv[8];
  load8(q + ((size_t)b * H + h) * D + sl * 8, qv);
  const float qscale = scale * 1.4426950408889634f;  // scores in log2 units
#pragma unroll
  for (int i = 0; i < 8; ++i) qv[i] *= qscale;

  float m = kNegBig, l = 0.f, acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;

  const int t_begin = split * chunk;
  const int t_end = min(ctx, t_begin + chunk);
  const size_t tok_stride = (size_t)Hkv * D;
  const int32_t* table = bt + (size_t)b * bt_stride;
  for (int t0 = t_begin + stream; t0 < t_end; t0 += C::kStreams * kUnroll) {
    float kv[kUnroll][8], vv[kUnroll][8];
    bool valid[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int t = t0 + u * C::kStreams;
      valid[u] = t < t_end;
      if (valid[u]) {
        const int blk = table[t / block_size];
        if (blk < 0 || blk >= num_blocks) {
          valid[u] = false;
          flag_bad_index(status);
        } else {
          const size_t off = ((size_t)blk * block_size + (t % block_size)) * tok_stride + (size_t)kvh * D + sl * 8;
          load8(kc + off, kv[u]);
          load8(vc + off, vv[u]);
        }
      }
    }
    float sc[kUnroll];
    float mnew = m;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      float d = 0.f;
      if (valid[u]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) d = fmaf(qv[i], kv[u][i], d);
      }
#pragma unroll
      for (int o = C::kLanesPerTok / 2; o > 0; o >>= 1) d += __shfl_xor_sync(grp_mask, d, o);
      sc[u] = valid[u] ? d : -INFINITY;
      mnew = fmaxf(mnew, sc[u]);
    }
    const float alpha = exp2f(m - mnew);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= alpha;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const float pu = exp2f(sc[u] - mnew);
      l += pu;
      if (valid[u]) {
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(pu, vv[u][i], acc[i]);
      }
    }
    m = mnew;
  }

  // merge the token streams of this CTA
  __shared__ float s_acc[C::kStreams][D];
  __shared__ float s_m[C::kStreams], s_l[C::kStreams];
  __shared__ int s_last;
#pragma unroll
  for (int i = 0; i < 8; ++i) s_acc[stream][sl * 8 + i] = acc[i];
  if (sl == 0) {
    s_m[stream] = m;
    s_l[stream] = l;
  }
  __syncthreads();
  const size_t ph = ((size_t)b * H + h);
  const size_t pidx = ph * n_splits + split;
  if (tid < D) {
    float mm = kNegBig;
    for (int s = 0; s < C::kStreams; ++s) mm = fmaxf(mm, s_m[s]);
    float ll = 0.f, aa = 0.f;
    for (int s = 0; s < C::kStreams; ++s) {
      const float w = exp2f(s_m[s] - mm);
      ll += s_l[s] * w;
      aa += s_acc[s][tid] * w;
    }
    __stcg(part_acc + pidx * D + tid, aa);
    if (tid == 0) {
      __stcg(part_ml + pidx * 2, mm);
      __stcg(part_ml + pidx * 2 + 1, ll);
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int prev = atomicAdd(counters + ph, 1);
    s_last = (prev + 1 == active);
    __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // last CTA of (b, h): merge `active` splits
  if (tid < D) {
    float mm = kNegBig;
    for (int s = 0; s < active; ++s) mm = fmaxf(mm, __ldcg(part_ml + (ph * n_splits + s) * 2));
    float ll = 0.f, aa = 0.f;
    for (int s = 0; s < active; ++s) {
      const size_t pi = ph * n_splits + s;
      const float w = exp2f(__ldcg(part_ml + pi * 2) - mm);
      ll += __ldcg(part_ml + pi * 2 + 1) * w;
      aa += __ldcg(part_acc + pi * D + tid) * w;
      __stcg(part_acc + pi * D + tid, 0.f);
    }
    out[ph * D + tid] = __float2half_rn(ll > 0.f ? aa / ll : 0.f);
  }
  __syncthreads();  // every thread has read part_ml before it is cleared
  // leave the whole workspace zero: its layout depends on the call's shape
  for (int i = tid; i < 2 * active; i += kAttnThreads) __stcg(part_ml + ph * n_splits * 2 + i, 0.f);
  if (tid == 0) counters[ph] = 0;
}

constexpr int kChunk = 256;

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
  store_kv_kernel<<<T, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(key), static_cast<const __half*>(value), ld_tok, Hkv * D, slot_mapping,
      static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), (long long)num_blocks * block_size,
      device_status_ptr());
  return launch_status("npl_store_kv");
}

extern "C" int npl_rope_store_kv(const void* qkv, int ld_qkv, int T, int H, int Hkv, int D, const void* cos_table,
                                 const void* sin_table, int max_position, const int64_t* positions,
                                 const int32_t* slot_mapping, void* q_out, void* k_cache, void* v_cache,
                                 int num_blocks, int block_size, void* stream) {
  if (int rc = check_device()) return rc;
  if (!qkv || !cos_table || !sin_table || !positions || !slot_mapping || !q_out || !k_cache || !v_cache)
    return fail(NPL_ERR_ARG, "npl_rope_store_kv: null pointer");
  if (T < 0 || H <= 0 || Hkv <= 0 || H % Hkv || D <= 0 || D % 2 || ld_qkv < (H + 2 * Hkv) * D ||
      max_position <= 0 || num_blocks <= 0 || block_size <= 0)
    return fail(NPL_ERR_ARG, "npl_rope_store_kv: bad shape");
  if (T == 0) return NPL_OK;
  rope_store_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(qkv), ld_qkv, H, Hkv, D, static_cast<const __half*>(cos_table),
      static_cast<const __half*>(sin_table), max_position, positions, slot_mapping, static_cast<__half*>(q_out),
      static_cast<__half*>(k_cache), static_cast<__half*>(v_cache), (long long)num_blocks * block_size,
      device_status_ptr());
  return launch_status("npl_rope_store_kv");
}

static int attn_splits(int max_blocks, int block_size) {
  const long long max_ctx = (long long)max_blocks * block_size;
  return (int)std::max<long long>(1, (max_ctx + kChunk - 1) / kChunk);
}

extern "C" size_t npl_decode_attention_workspace_bytes(int B, int H, int D, int max_blocks, int block_size) {
  if (B <= 0 || H <= 0 || D <= 0 || max_blocks <= 0 || block_size <= 0) return 0;
  const size_t parts = (size_t)B * H * attn_splits(max_blocks, block_size);
  const size_t ml = (parts * 2 * sizeof(float) + 255) & ~size_t(255);
  const size_t acc = (parts * D * sizeof(float) + 255) & ~size_t(255);
  const size_t cnt = ((size_t)B * H * sizeof(int32_t) + 255) & ~size_t(255);
  return ml + acc + cnt;
}

extern "C" int npl_paged_decode_attention(const void* q, int B, int H, int Hkv, int D, const void* k_cache,
                                          const void* v_cache, int num_blocks, int block_size,
                                          const int32_t* block_tables, int bt_stride, int max_blocks,
                                          const int32_t* context_lens, float scale, void* out, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  if (int rc = check_device()) return rc;
  if (!q || !k_cache || !v_cache || !block_tables || !context_lens || !out)
    return fail(NPL_ERR_ARG, "npl_paged_decode_attention: null pointer");
  if (B < 0 || H <= 0 || Hkv <= 0 || H % Hkv || num_blocks <= 0 || block_size <= 0 || max_blocks <= 0 ||
      bt_stride < max_blocks)
    return fail(NPL_ERR_ARG, "npl_paged_decode_attention: bad shape");
  if (D != 128 && D != 64) return fail(NPL_ERR_UNSUPPORTED, "npl_paged_decode_attention: head_dim %d (64 or 128)", D);
  for (const void* p : std::initializer_list<const void*>{q, k_cache, v_cache})
    if (!aligned16(p)) return fail(NPL_ERR_ARG, "npl_paged_decode_attention: pointers must be 16-byte aligned");
  if (B == 0) return NPL_OK;
  const size_t need = npl_decode_attention_workspace_bytes(B, H, D, max_blocks, block_size);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(NPL_ERR_ARG, "npl_paged_decode_attention: workspace of %zu bytes required", need);
  const int splits = attn_splits(max_blocks, block_size);
  const size_t parts = (size_t)B * H * splits;
  char* ws = static_cast<char*>(workspace);
  float* part_ml = reinterpret_cast<float*>(ws);
  float* part_acc = reinterpret_cast<float*>(ws + ((parts * 2 * sizeof(float) + 255) & ~size_t(255)));
  int32_t* counters = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(part_acc) +
                                                 ((parts * D * sizeof(float) + 255) & ~size_t(255)));
  dim3 grid(splits, H, B);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128)
    decode_attn_kernel<128><<<grid, kAttnThreads, 0, st>>>(
        static_cast<const __half*>(q), H, Hkv, static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
        num_blocks, block_size, block_tables, bt_stride, max_blocks, context_lens, scale, kChunk,
        static_cast<__half*>(out),
        part_ml, part_acc, counters, device_status_ptr());
  else
    decode_attn_kernel<64><<<grid, kAttnThreads, 0, st>>>(
        static_cast<const __half*>(q), H, Hkv, static_cast<const __half*>(k_cache), static_cast<const __half*>(v_cache),
        num_blocks, block_size, block_tables, bt_stride, max_blocks, context_lens, scale, kChunk,
        static_cast<__half*>(out),
        part_ml, part_acc, counters, device_status_ptr());
  return launch_status("npl_paged_decode_attention");
}
