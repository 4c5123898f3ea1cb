// Per-row dynamic int8 quantisation and fused RMSNorm + quantisation.
//
// npl_quant_rows     <- w8a8.py:33-50,106-115 (and :53-62 applied to weight rows)
// npl_rmsnorm_quant  <- lightweight_runner.py:239-260 (eager RMSNorm / residual_norm)
//                       followed by w8a8.py:106-115
// npl_row_absmax, npl_quant_rows_absmax, npl_dequant
//                    <- w8a8.py:106-115 and :118-139 split at the reductions a
//                       tensor-parallel layer needs: the per-token absmax (max
//                       over ranks) before quantising, and the int32
//                       accumulator (sum over ranks) before dequantising
//
// One CTA per row; rows are short (decode: M <= 64 rows of 4096 or 11008), so
// both kernels are latency-bound single passes over L2-resident data.
#include <algorithm>
#include <initializer_list>

#include "npl_common.cuh"

namespace npl {
namespace {

// Threads per row: a decode row (4096 or 11008 columns) takes one or two
// 16-byte loads per thread, issued together, so a row costs about one L2
// round trip per pass instead of one per 2048 columns.
constexpr int kQuantThreads = 1024;
constexpr int kNormThreads = 512;

template <typename T>
struct Vec;  // 16-byte vector of T
template <>
struct Vec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float (&v)[4]) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  }
};
template <>
struct Vec<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float (&v)[8]) {
    const uint4 x = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};

template <int N>
__device__ __forceinline__ void store_q(int8_t* dst, const int (&q)[N]);
template <>
__device__ __forceinline__ void store_q<4>(int8_t* dst, const int (&q)[4]) {
  char4 c = make_char4((char)q[0], (char)q[1], (char)q[2], (char)q[3]);
  *reinterpret_cast<char4*>(dst) = c;
}
template <>
__device__ __forceinline__ void store_q<8>(int8_t* dst, const int (&q)[8]) {
  uint2 u;
  u.x = (uint32_t)(q[0] & 0xff) | ((uint32_t)(q[1] & 0xff) << 8) | ((uint32_t)(q[2] & 0xff) << 16) |
        ((uint32_t)(q[3] & 0xff) << 24);
  u.y = (uint32_t)(q[4] & 0xff) | ((uint32_t)(q[5] & 0xff) << 8) | ((uint32_t)(q[6] & 0xff) << 16) |
        ((uint32_t)(q[7] & 0xff) << 24);
  *reinterpret_cast<uint2*>(dst) = u;
}

// absmax_in (float bits, optional): use this per-row absmax instead of the
// row's own; absmax_out (optional): record the row's absmax; q == null:
// record the absmax only. A CTA handles R consecutive rows (R > 1 for long
// batches, so that an SM keeps more rows in flight); each thread reads the
// same chunks of every row, and a max does not depend on its order, so the
// result is the same for any R.
template <typename T, int R>
__global__ void __launch_bounds__(kQuantThreads) quant_rows_kernel(const T* __restrict__ x, int rows, int cols,
                                                                   int ldx, int8_t* __restrict__ q, int ldq,
                                                                   float* __restrict__ scale,
                                                                   const int32_t* __restrict__ absmax_in,
                                                                   int32_t* __restrict__ absmax_out) {
  __shared__ float red[R][32];
  constexpr int V = Vec<T>::N;
  pdl_wait();
  const int r0 = blockIdx.x * R;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float amax[R];
#pragma unroll
  for (int r = 0; r < R; ++r) amax[r] = 0.f;
  if (absmax_in) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (r0 + r < rows) amax[r] = __int_as_float(absmax_in[r0 + r]);
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r0 + r >= rows) continue;
      const T* row = x + (size_t)(r0 + r) * ldx;
#pragma unroll 2
      for (int c = threadIdx.x * V; c < cols; c += kQuantThreads * V) {
        float v[V];
        Vec<T>::load(row + c, v);
#pragma unroll
        for (int i = 0; i < V; ++i) amax[r] = fmaxf(amax[r], fabsf(v[i]));
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      amax[r] = warp_max(amax[r]);
      if (lane == 0) red[r][warp] = amax[r];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) amax[r] = warp_max(lane < kQuantThreads / 32 ? red[r][lane] : 0.f);
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (absmax_out && threadIdx.x == 0 && r0 + r < rows) absmax_out[r0 + r] = __float_as_int(amax[r]);
  if (!q) {
    pdl_trigger();
    return;
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (r0 + r >= rows) continue;
    const float s = scale_from_absmax(amax[r]);
    const float rs = quant_recip(s);
    if (threadIdx.x == 0) scale[r0 + r] = s;
    const T* row = x + (size_t)(r0 + r) * ldx;
    int8_t* qrow = q + (size_t)(r0 + r) * ldq;
#pragma unroll 2
    for (int c = threadIdx.x * V; c < cols; c += kQuantThreads * V) {
      float v[V];
      Vec<T>::load(row + c, v);
      int qi[V];
#pragma unroll
      for (int i = 0; i < V; ++i) qi[i] = quantize_one(v[i], s, rs);
      store_q<V>(qrow + c, qi);
    }
  }
  pdl_trigger_after_writes();  // the rows may be weights, read by the next linear before its pdl_wait
}

// RMSNorm of one fp16 row (optionally x + residual) + per-token quantisation.
// The row is staged in shared memory as fp16.
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_quant_kernel(const __half* __restrict__ x, const __half* __restrict__ res,
                         const __half* __restrict__ w, float eps, int cols, __half* __restrict__ sum_out,
                         __half* __restrict__ normed_out, int8_t* __restrict__ q, float* __restrict__ scale) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* srow = reinterpret_cast<__half*>(smem_raw);
  __shared__ double dred[32];
  __shared__ float fred[32];
  pdl_wait();
  pdl_trigger();
  const size_t base = (size_t)blockIdx.x * cols;

  // 1. s = x (+ residual, fp16 add), sum of squares in fp64 (squares of fp16
  //    values are exact in fp32 and fp64).
  double ss = 0.0;
#pragma unroll 2
  for (int c = threadIdx.x * 8; c < cols; c += kNormThreads * 8) {
    float v[8];
    Vec<__half>::load(x + base + c, v);
    if (res) {
      float r[8];
      Vec<__half>::load(res + base + c, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __half2float(__float2half_rn(__fadd_rn(v[i], r[i])));
    }
    uint4 packed;
    __half2* hp = reinterpret_cast<__half2*>(&packed);
#pragma unroll
    for (int i = 0; i < 4; ++i) hp[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(srow + c) = packed;
    if (res && sum_out) *reinterpret_cast<uint4*>(sum_out + base + c) = packed;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += (double)v[i] * (double)v[i];
  }
  ss = block_sum(ss, dred);
  // mean rounded once to fp32; + eps; IEEE 1/sqrt (torch.rsqrt on CPU).
  const float mean = __double2float_rn(ss / (double)cols);
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));

  // 2. n = fp16(w * fp16(s * r)); absmax of n.
  float amax = 0.f;
  for (int c = threadIdx.x * 8; c < cols; c += kNormThreads * 8) {
    float v[8], wv[8];
    Vec<__half>::load(srow + c, v);
    Vec<__half>::load(w + c, wv);
    uint4 packed;
    __half* hp = reinterpret_cast<__half*>(&packed);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float y = __half2float(__float2half_rn(__fmul_rn(v[i], r)));
      hp[i] = __float2half_rn(__fmul_rn(wv[i], y));
      amax = fmaxf(amax, fabsf(__half2float(hp[i])));
    }
    *reinterpret_cast<uint4*>(srow + c) = packed;
    if (normed_out) *reinterpret_cast<uint4*>(normed_out + base + c) = packed;
  }
  amax = block_max(amax, fred);
  const float s = scale_from_absmax(amax);
  const float rs = quant_recip(s);
  if (threadIdx.x == 0) scale[blockIdx.x] = s;

  // 3. quantise (each thread re-reads only the chunks it wrote).
  for (int c = threadIdx.x * 8; c < cols; c += kNormThreads * 8) {
    float v[8];
    Vec<__half>::load(srow + c, v);
    int qi[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) qi[i] = quantize_one(v[i], s, rs);
    store_q<8>(q + base + c, qi);
  }
}

// quantize_symmetric with a caller-given scale (w8a8.py:33-43): one fp32
// scale per row (scale_stride 1) or one for the whole tensor (stride 0),
// q = clamp(rint(v / s), -127, 127) with the IEEE quotient of every element
// (the given scale need not be an fp16 value, so no reciprocal shortcut).
// Grid (rows, ceil(cols / 2048)), 256 threads x 8 elements.
template <typename T>
__global__ void __launch_bounds__(256) quant_given_scale_kernel(const T* __restrict__ x, int cols, int ldx,
                                                                const float* __restrict__ scale, int scale_stride,
                                                                int8_t* __restrict__ q, int ldq) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const float s = scale[(size_t)r * scale_stride];
  const T* row = x + (size_t)r * ldx;
  int8_t* qrow = q + (size_t)r * ldq;
  const int c0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (c0 >= cols) return;
  float v[8];
  if constexpr (Vec<T>::N == 8) {
    Vec<T>::load(row + c0, v);
  } else {
    float a[4], b[4];
    Vec<T>::load(row + c0, a);
    Vec<T>::load(row + c0 + 4, b);
#pragma unroll
    for (int i = 0; i < 4; ++i) { v[i] = a[i]; v[4 + i] = b[i]; }
  }
  int qi[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) qi[i] = max(-127, min(127, __float2int_rn(__fdiv_rn(v[i], s))));
  store_q<8>(qrow + c0, qi);
}

// Dequantisation of int8 rows: out = fp32(q) * s (one fp32 rounding), stored
// as out_dtype; the QDQ value of w8a8.py:53-62 (per_output_weight_qdq) and
// :101-103,106-115 (static / dynamic activation QDQ). Same grid as above.
__global__ void __launch_bounds__(256) dequant_rows_kernel(const int8_t* __restrict__ q, int cols, int ldq,
                                                           const float* __restrict__ scale, int scale_stride,
                                                           void* __restrict__ out, int ld_out, int out_dtype) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const float s = scale[(size_t)r * scale_stride];
  const int c0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (c0 >= cols) return;
  const uint2 packed = *reinterpret_cast<const uint2*>(q + (size_t)r * ldq + c0);
  const int8_t* b = reinterpret_cast<const int8_t*>(&packed);
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __fmul_rn((float)b[i], s);
  if (out_dtype == NPL_F32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)r * ld_out + c0);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    uint4 h;
    __half2* hp = reinterpret_cast<__half2*>(&h);
#pragma unroll
    for (int i = 0; i < 4; ++i) hp[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(static_cast<__half*>(out) + (size_t)r * ld_out + c0) = h;
  }
}

// scale_from_absmax (w8a8.py:46-50) elementwise over n fp32 values.
__global__ void __launch_bounds__(256) scale_from_absmax_kernel(const float* __restrict__ absmax, int n,
                                                                float* __restrict__ scale) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i < n) scale[i] = scale_from_absmax(absmax[i]);
}

// out[m, n] = ((acc * sa[m]) * sw[n]) + bias[n], as the linear's epilogue
// (NPL_EPI_NONE to out_dtype; NPL_EPI_RESIDUAL: fp16(fp16(v) + residual)).
// Grid (M, ceil(N / 256)), one element per thread.
__global__ void __launch_bounds__(256) dequant_kernel(const int32_t* __restrict__ acc, int ld_acc,
                                                      const float* __restrict__ sa, const float* __restrict__ sw,
                                                      const float* __restrict__ bias, int N, int epilogue,
                                                      const __half* __restrict__ residual, int ld_res, void* out,
                                                      int ld_out, int out_dtype) {
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x, n = blockIdx.y * 256 + threadIdx.x;
  if (n >= N) return;
  float v = __fmul_rn(__fmul_rn(__int2float_rn(acc[(size_t)m * ld_acc + n]), sa[m]), sw[n]);
  if (bias) v = __fadd_rn(v, bias[n]);
  if (epilogue == NPL_EPI_RESIDUAL) {
    const float o = __half2float(__float2half_rn(v));
    const float r = __half2float(residual[(size_t)m * ld_res + n]);
    static_cast<__half*>(out)[(size_t)m * ld_out + n] = __float2half_rn(__fadd_rn(o, r));
  } else if (out_dtype == NPL_F32) {
    static_cast<float*>(out)[(size_t)m * ld_out + n] = v;
  } else {
    static_cast<__half*>(out)[(size_t)m * ld_out + n] = __float2half_rn(v);
  }
}

}  // namespace
}  // namespace npl

using namespace npl;

namespace npl {
namespace {

int quant_rows_common(const char* what, const void* x, int x_dtype, int rows, int cols, int ldx,
                      const int32_t* absmax_in, int32_t* absmax_out, int8_t* q, int ldq, float* scale,
                      void* stream) {
  if (int rc = check_device()) return rc;
  if (!x || (q && !scale)) return fail(NPL_ERR_ARG, "%s: null pointer", what);
  if (rows < 0 || cols <= 0 || cols % 16 || ldx < cols || ldx % 16 || (q && (ldq < cols || ldq % 16)))
    return fail(NPL_ERR_ARG, "%s: bad shape rows=%d cols=%d ldx=%d ldq=%d", what, rows, cols, ldx, ldq);
  if (!aligned16(x) || (q && !aligned16(q))) return fail(NPL_ERR_ARG, "%s: pointers must be 16-byte aligned", what);
  if (rows == 0) return NPL_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // decode batches: a CTA per row; longer batches: 4 rows per CTA
  const bool multi = rows > 64;
  const dim3 grid(multi ? (rows + 3) / 4 : rows);
  if (x_dtype == NPL_F32)
    return launch_pdl(what, multi ? quant_rows_kernel<float, 4> : quant_rows_kernel<float, 1>, grid,
                      dim3(kQuantThreads), 0, st, static_cast<const float*>(x), rows, cols, ldx, q, ldq, scale,
                      absmax_in, absmax_out);
  if (x_dtype == NPL_F16)
    return launch_pdl(what, multi ? quant_rows_kernel<__half, 4> : quant_rows_kernel<__half, 1>, grid,
                      dim3(kQuantThreads), 0, st, static_cast<const __half*>(x), rows, cols, ldx, q, ldq, scale,
                      absmax_in, absmax_out);
  return fail(NPL_ERR_ARG, "%s: x_dtype must be NPL_F32 or NPL_F16", what);
}

}  // namespace
}  // namespace npl

extern "C" int npl_quant_rows(const void* x, int x_dtype, int rows, int cols, int ldx, int8_t* q, int ldq,
                              float* scale, void* stream) {
  if (!q) return fail(NPL_ERR_ARG, "npl_quant_rows: null pointer");
  return quant_rows_common("npl_quant_rows", x, x_dtype, rows, cols, ldx, nullptr, nullptr, q, ldq, scale, stream);
}

extern "C" int npl_row_absmax(const void* x, int x_dtype, int rows, int cols, int ldx, int32_t* absmax_out,
                              void* stream) {
  if (!absmax_out) return fail(NPL_ERR_ARG, "npl_row_absmax: null pointer");
  return quant_rows_common("npl_row_absmax", x, x_dtype, rows, cols, ldx, nullptr, absmax_out, nullptr, 0, nullptr,
                           stream);
}

extern "C" int npl_quant_rows_absmax(const void* x, int x_dtype, int rows, int cols, int ldx,
                                     const int32_t* absmax_in, int8_t* q, int ldq, float* scale, void* stream) {
  if (!absmax_in || !q) return fail(NPL_ERR_ARG, "npl_quant_rows_absmax: null pointer");
  return quant_rows_common("npl_quant_rows_absmax", x, x_dtype, rows, cols, ldx, absmax_in, nullptr, q, ldq, scale,
                           stream);
}

extern "C" int npl_quant_given_scale(const void* x, int x_dtype, int rows, int cols, int ldx, const float* scale,
                                     int scale_stride, int8_t* q, int ldq, void* stream) {
  if (int rc = check_device()) return rc;
  if (!x || !scale || !q) return fail(NPL_ERR_ARG, "npl_quant_given_scale: null pointer");
  if (rows < 0 || cols <= 0 || cols % 16 || ldx < cols || ldx % 16 || ldq < cols || ldq % 16 ||
      (scale_stride != 0 && scale_stride != 1))
    return fail(NPL_ERR_ARG, "npl_quant_given_scale: bad shape rows=%d cols=%d ldx=%d ldq=%d scale_stride=%d", rows,
                cols, ldx, ldq, scale_stride);
  if (!aligned16(x) || !aligned16(q)) return fail(NPL_ERR_ARG, "npl_quant_given_scale: pointers must be 16-byte aligned");
  if (rows == 0) return NPL_OK;
  const dim3 grid(rows, (cols + 2047) / 2048);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == NPL_F32)
    return launch_pdl("npl_quant_given_scale", quant_given_scale_kernel<float>, grid, dim3(256), 0, st,
                      static_cast<const float*>(x), cols, ldx, scale, scale_stride, q, ldq);
  if (x_dtype == NPL_F16)
    return launch_pdl("npl_quant_given_scale", quant_given_scale_kernel<__half>, grid, dim3(256), 0, st,
                      static_cast<const __half*>(x), cols, ldx, scale, scale_stride, q, ldq);
  return fail(NPL_ERR_ARG, "npl_quant_given_scale: x_dtype must be NPL_F32 or NPL_F16");
}

extern "C" int npl_dequant_rows(const int8_t* q, int rows, int cols, int ldq, const float* scale, int scale_stride,
                                void* out, int ld_out, int out_dtype, void* stream) {
  if (int rc = check_device()) return rc;
  if (!q || !scale || !out) return fail(NPL_ERR_ARG, "npl_dequant_rows: null pointer");
  if (rows < 0 || cols <= 0 || cols % 16 || ldq < cols || ldq % 16 || ld_out < cols || ld_out % 16 ||
      (scale_stride != 0 && scale_stride != 1) || (out_dtype != NPL_F32 && out_dtype != NPL_F16))
    return fail(NPL_ERR_ARG, "npl_dequant_rows: bad shape rows=%d cols=%d ldq=%d ld_out=%d", rows, cols, ldq,
                ld_out);
  if (!aligned16(q) || !aligned16(out)) return fail(NPL_ERR_ARG, "npl_dequant_rows: pointers must be 16-byte aligned");
  if (rows == 0) return NPL_OK;
  return launch_pdl("npl_dequant_rows", dequant_rows_kernel, dim3(rows, (cols + 2047) / 2048), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), q, cols, ldq, scale, scale_stride, out, ld_out, out_dtype);
}

// act_fn(gate) * up on fp16 rows (lightweight_runner.py:358, the unfused MLP):
// out = fp16(silu_f16(g) * u), the same arithmetic as the SiLU * up epilogue
// of npl_w8a8_linear_ex. 8 columns per thread.
__global__ void __launch_bounds__(256) silu_mul_kernel(const __half* __restrict__ gate, int ld_gate,
                                                       const __half* __restrict__ up, int ld_up, int cols,
                                                       __half* __restrict__ out, int ld_out) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  const int c0 = (blockIdx.y * 256 + threadIdx.x) * 8;
  if (c0 >= cols) return;
  const uint4 g8 = *reinterpret_cast<const uint4*>(gate + (size_t)r * ld_gate + c0);
  const uint4 u8 = *reinterpret_cast<const uint4*>(up + (size_t)r * ld_up + c0);
  const __half* g = reinterpret_cast<const __half*>(&g8);
  const __half* u = reinterpret_cast<const __half*>(&u8);
  uint4 o8;
  __half* o = reinterpret_cast<__half*>(&o8);
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = __float2half_rn(__fmul_rn(silu_f16(__half2float(g[i])), __half2float(u[i])));
  *reinterpret_cast<uint4*>(out + (size_t)r * ld_out + c0) = o8;
}

extern "C" int npl_silu_mul(const void* gate, int ld_gate, const void* up, int ld_up, int rows, int cols, void* out,
                            int ld_out, void* stream) {
  if (int rc = check_device()) return rc;
  if (!gate || !up || !out) return fail(NPL_ERR_ARG, "npl_silu_mul: null pointer");
  if (rows < 0 || cols <= 0 || cols % 8 || ld_gate < cols || ld_gate % 8 || ld_up < cols || ld_up % 8 ||
      ld_out < cols || ld_out % 8)
    return fail(NPL_ERR_ARG, "npl_silu_mul: bad shape rows=%d cols=%d ld_gate=%d ld_up=%d ld_out=%d", rows, cols,
                ld_gate, ld_up, ld_out);
  if (!aligned16(gate) || !aligned16(up) || !aligned16(out))
    return fail(NPL_ERR_ARG, "npl_silu_mul: pointers must be 16-byte aligned");
  if (rows == 0) return NPL_OK;
  return launch_pdl("npl_silu_mul", silu_mul_kernel, dim3(rows, (cols + 2047) / 2048), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __half*>(gate), ld_gate,
                    static_cast<const __half*>(up), ld_up, cols, static_cast<__half*>(out), ld_out);
}

extern "C" int npl_scale_from_absmax(const float* absmax, int n, float* scale, void* stream) {
  if (int rc = check_device()) return rc;
  if (!absmax || !scale || n < 0) return fail(NPL_ERR_ARG, "npl_scale_from_absmax: bad arguments");
  if (n == 0) return NPL_OK;
  return launch_pdl("npl_scale_from_absmax", scale_from_absmax_kernel, dim3((n + 255) / 256), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), absmax, n, scale);
}

extern "C" int npl_dequant(const int32_t* acc, int ld_acc, const float* sa, const float* sw, const float* bias,
                           int M, int N, int epilogue, const void* residual, int ld_res, void* out, int ld_out,
                           int out_dtype, void* stream) {
  if (int rc = check_device()) return rc;
  if (!acc || !sa || !sw || !out) return fail(NPL_ERR_ARG, "npl_dequant: null pointer");
  if (M < 0 || N <= 0 || ld_acc < N || ld_out < N)
    return fail(NPL_ERR_ARG, "npl_dequant: bad shape M=%d N=%d", M, N);
  if (epilogue == NPL_EPI_RESIDUAL) {
    if (!residual || ld_res < N || out_dtype != NPL_F16)
      return fail(NPL_ERR_ARG, "npl_dequant: the residual epilogue needs an fp16 residual and fp16 out");
  } else if (epilogue != NPL_EPI_NONE || (out_dtype != NPL_F16 && out_dtype != NPL_F32)) {
    return fail(NPL_ERR_ARG, "npl_dequant: epilogue NPL_EPI_NONE (fp16/fp32 out) or NPL_EPI_RESIDUAL");
  }
  if (M == 0) return NPL_OK;
  return launch_pdl("npl_dequant", dequant_kernel, dim3(M, (N + 255) / 256), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), acc, ld_acc, sa, sw, bias, N, epilogue,
                    static_cast<const __half*>(residual), ld_res, out, ld_out, out_dtype);
}

extern "C" int npl_rmsnorm_quant(const void* x, const void* residual, const void* weight, float eps, int rows,
                                 int cols, void* sum_out, void* normed_out, int8_t* q, float* scale,
                                 void* stream) {
  if (int rc = check_device()) return rc;
  if (!x || !weight || !q || !scale) return fail(NPL_ERR_ARG, "npl_rmsnorm_quant: null pointer");
  if (rows < 0 || cols <= 0 || cols % 16 || cols > 48 * 1024)
    return fail(NPL_ERR_ARG, "npl_rmsnorm_quant: bad shape rows=%d cols=%d", rows, cols);
  for (const void* p : std::initializer_list<const void*>{x, residual, weight, sum_out, normed_out, (const void*)q})
    if (p && !aligned16(p)) return fail(NPL_ERR_ARG, "npl_rmsnorm_quant: pointers must be 16-byte aligned");
  if (rows == 0) return NPL_OK;
  const size_t smem = (size_t)cols * sizeof(__half);
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(rmsnorm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return launch_status("npl_rmsnorm_quant: smem attribute");
  }
  return launch_pdl("npl_rmsnorm_quant", rmsnorm_quant_kernel, dim3(rows), dim3(kNormThreads), smem,
                    static_cast<cudaStream_t>(stream), static_cast<const __half*>(x),
                    static_cast<const __half*>(residual), static_cast<const __half*>(weight), eps, cols,
                    static_cast<__half*>(sum_out), static_cast<__half*>(normed_out), q, scale);
}
