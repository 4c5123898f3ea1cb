/*
 * libnpl_w8a8 — C ABI of the B200 (sm_100a) W8A8 linear + paged-decode path.
 *
 * Every entry takes device pointers, sizes and strides (in elements unless a
 * name says bytes) and a CUDA stream passed as `void*` (a cudaStream_t; NULL
 * is the legacy default stream). Work is enqueued on that stream; no entry
 * synchronises the host, allocates or frees device memory. Apart from
 * npl_w8a8_linear_noalloc (see its own comment), every call can be recorded
 * into a CUDA graph. Buffers, including workspaces, belong to the caller.
 *
 * Return value: NPL_OK or an NPL_ERR_* code; npl_last_error_string() gives
 * the message (per host thread). Arguments are validated on the host before
 * any launch. Device-side waits are bounded (~1 s); a kernel that gives up
 * records a code in the per-device status word read by npl_device_status().
 *
 * Reference interfaces replaced (paths in the nanopointllm project):
 *   nanopointllm/compression/w8a8.py        the W8A8 numeric contract
 *   nanopointllm/llama/lightweight_runner.py RMSNorm / MLP / LM-head call sites
 *   nanopointllm/llama/paged_attention.py    QKV / O call sites, rotary_fn +
 *                                            store_kvcache, paged_decode_attention
 */
#ifndef NPL_W8A8_H_
#define NPL_W8A8_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NPL_OK 0
#define NPL_ERR_ARG 1         /* null pointer, bad shape, stride or alignment   */
#define NPL_ERR_OVERFLOW 2    /* K * 127^2 >= 2^31 (w8a8.py:152-153)             */
#define NPL_ERR_LAUNCH 3      /* CUDA launch / driver error                      */
#define NPL_ERR_TIMEOUT 4     /* a bounded device wait expired                   */
#define NPL_ERR_UNSUPPORTED 5 /* not an sm_100 device, or a shape outside scope  */

/* element types */
#define NPL_F32 0
#define NPL_F16 1

/* fused epilogues of npl_w8a8_linear / npl_w8a8_linear_ex */
#define NPL_EPI_NONE 0     /* out = dequant(acc)                                  */
#define NPL_EPI_RESIDUAL 1 /* out = fp16(fp16(dequant(acc)) + residual)           */
#define NPL_EPI_SILU_MUL 2 /* gate/up rows interleaved by 8; out = silu(g) * u    */
#define NPL_EPI_ROPE_KV 3  /* packed QKV: RoPE on q/k, q -> q_out, k/v -> cache (npl_w8a8_linear_ex) */

/* activation operand of npl_w8a8_linear_ex */
#define NPL_X_INT8 0        /* int8 [M, K] + fp32 per-token scales                       */
#define NPL_X_F16_ABSMAX 1  /* fp16 [M, K] quantised in the kernel with a given absmax   */
#define NPL_X_F16_RMSNORM 2 /* fp16 [M, K] RMSNorm-ed, then quantised in the kernel      */

const char* npl_last_error_string(void);
int npl_version(void);

/* Reads the per-device status word of the current device (synchronous; call
 * it outside stream capture). *code receives 0 or the NPL_DEV_* code of the
 * first expired wait; reset != 0 clears the word. Returns NPL_ERR_TIMEOUT
 * when a code was set. */
int npl_device_status(int* code, int reset);

/*
 * Per-row dynamic symmetric int8 quantisation (rows x cols, row stride ldx):
 *   scale[r] = fp32(fp16(max(absmax_r, fp16.tiny) / 127)) (>= fp16.tiny)
 *   q[r, c]  = clamp(rint(x / scale[r]), -127, 127)
 * Replaces w8a8.py:33-43 quantize_symmetric + :46-50 scale_from_absmax, as
 * used per token by :106-115 dynamic_per_token_activation_qdq and per output
 * channel by :53-62 per_output_weight_qdq. x_dtype is NPL_F32 or NPL_F16.
 * cols, ldx, ldq multiples of 16; pointers 16-byte aligned.
 */
int npl_quant_rows(const void* x, int x_dtype, int rows, int cols, int ldx, int8_t* q, int ldq,
                   float* scale, void* stream);

/*
 * The two halves of npl_quant_rows, for a tensor-parallel layer whose input
 * rows are split over ranks (the per-token scale needs the absmax of the
 * whole row, a max over ranks; no counterpart in the reference, which runs on
 * one device):
 *   npl_row_absmax:        absmax_out[r] = max |x[r, :]| as fp32 bits (int32)
 *   npl_quant_rows_absmax: scale and q as npl_quant_rows, from the given
 *                          absmax_in[r] (fp32 bits) instead of the row's own
 * Same shape and alignment rules as npl_quant_rows.
 */
int npl_row_absmax(const void* x, int x_dtype, int rows, int cols, int ldx, int32_t* absmax_out, void* stream);
int npl_quant_rows_absmax(const void* x, int x_dtype, int rows, int cols, int ldx, const int32_t* absmax_in,
                          int8_t* q, int ldq, float* scale, void* stream);

/*
 * quantize_symmetric with a caller-given fp32 scale (w8a8.py:33-43, the
 * static per-tensor mode of :94-103 and any precomputed per-token scale):
 *   q[r, c] = clamp(rint(x[r, c] / scale[r * scale_stride]), -127, 127)
 * with the IEEE fp32 quotient; scale_stride 1 = one scale per row, 0 = one
 * scale for the whole tensor. The caller checks scale > 0 (the reference
 * raises ValueError). Same shape and alignment rules as npl_quant_rows.
 */
int npl_quant_given_scale(const void* x, int x_dtype, int rows, int cols, int ldx, const float* scale,
                          int scale_stride, int8_t* q, int ldq, void* stream);

/*
 * QDQ values of int8 rows: out[r, c] = fp32(q[r, c]) * scale[r * scale_stride]
 * stored as out_dtype (NPL_F32, or NPL_F16 rounded once): the dequantised
 * weight of w8a8.py:53-62 per_output_weight_qdq and the activation QDQ of
 * :101-103 static_activation_qdq / :106-115 dynamic_per_token_activation_qdq.
 * cols, ldq, ld_out multiples of 16; pointers 16-byte aligned.
 */
int npl_dequant_rows(const int8_t* q, int rows, int cols, int ldq, const float* scale, int scale_stride, void* out,
                     int ld_out, int out_dtype, void* stream);

/*
 * act_fn(gate) * up of the unfused MLP on fp16 rows (lightweight_runner.py:358):
 *   out[r, c] = fp16(fp16(silu(gate[r, c])) * up[r, c])
 * with SiLU rounded once to fp16 from the exact value, the arithmetic of the
 * SiLU * up epilogue of npl_w8a8_linear_ex (NPL_EPI_SILU_MUL). cols and the
 * leading dimensions multiples of 8; pointers 16-byte aligned.
 */
int npl_silu_mul(const void* gate, int ld_gate, const void* up, int ld_up, int rows, int cols, void* out, int ld_out,
                 void* stream);

/*
 * scale_from_absmax (w8a8.py:46-50) over n fp32 absmax values:
 *   scale[i] = max(fp32(fp16(max(absmax[i], fp16.tiny) / 127)), fp16.tiny)
 */
int npl_scale_from_absmax(const float* absmax, int n, float* scale, void* stream);

/*
 * Dequantisation of int32 accumulators, as the epilogue of npl_w8a8_linear
 * (w8a8.py:118-139): v = ((acc[m, n] * sa[m]) * sw[n]) (+ bias[n]);
 * NPL_EPI_NONE writes v as out_dtype, NPL_EPI_RESIDUAL writes
 * fp16(fp16(v) + residual[m, n]). For a row-parallel linear whose int32
 * partial accumulators were summed over ranks (no counterpart in the
 * reference).
 */
int npl_dequant(const int32_t* acc, int ld_acc, const float* sa, const float* sw, const float* bias_or_null,
                int M, int N, int epilogue, const void* residual_or_null, int ld_res, void* out, int ld_out,
                int out_dtype, void* stream);

/*
 * Fused RMSNorm + per-token int8 quantisation of fp16 rows (contiguous):
 *   s = residual ? fp16(x + residual) : x            (sum_out <- s if given)
 *   n = fp16(w * fp16(s * 1/sqrt(mean(s^2) + eps)))  (normed_out <- n if given)
 *   q, scale = per-row quantisation of n             (as npl_quant_rows)
 * Replaces lightweight_runner.py:239-260 (LightweightRMSNorm.forward /
 * residual_norm, eager semantics) followed by w8a8.py:106-115. mean(s^2) is
 * the fp64 sum of the squares divided by cols, rounded once to fp32.
 */
int npl_rmsnorm_quant(const void* x, const void* residual_or_null, const void* weight, float eps,
                      int rows, int cols, void* sum_out_or_null, void* normed_out_or_null, int8_t* q,
                      float* scale, void* stream);

/*
 * W8A8 linear: acc[m, n] = sum_k qa[m, k] * qw[n, k] (int32, exact), then
 *   v = ((float)acc * sa[m]) * sw[n] (+ bias[n]), each step an fp32 rounding,
 * and the epilogue:
 *   NPL_EPI_NONE      out[m, n] = v as out_dtype (NPL_F32 or NPL_F16)
 *   NPL_EPI_RESIDUAL  out[m, n] = fp16(fp16(v) + residual[m, n])       (fp16)
 *   NPL_EPI_SILU_MUL  rows of qw are packed in groups of 16: group j holds
 *                     gate rows [8j, 8j+8) then the matching 8 up rows; out
 *                     is [M, N/2] fp16 with out[m, i] = fp16(silu(g) * u),
 *                     g = fp16(v_gate), u = fp16(v_up), silu(g) = g / (1 +
 *                     exp(-g)) rounded once to fp16 from the exact value.
 * acc_out_or_null receives the int32 accumulators [M, N] (row stride N).
 * Replaces w8a8.py:118-139 integer_linear_per_output_reference and the
 * projection call sites paged_attention.py:97-124,283-305,1349-1352,1488 and
 * lightweight_runner.py:320-404,675-681 (F.linear on packed QKV, O, packed
 * gate/up + act_fn(gate)*up, down, LM head).
 * K multiple of 16 and K*127^2 < 2^31; lda, ldw multiples of 16; int8
 * operands 16-byte aligned. The workspace (npl_linear_workspace_bytes) must be
 * zero-filled once by the caller; every call leaves it zeroed again. Calls
 * that share a workspace must be ordered on one stream.
 */
size_t npl_linear_workspace_bytes(int M, int N, int K);
int npl_w8a8_linear(const int8_t* qa, int lda, const float* sa, const int8_t* qw, int ldw,
                    const float* sw, const float* bias_or_null, int M, int N, int K, int epilogue,
                    const void* residual_or_null, int ld_res, void* out, int ld_out, int out_dtype,
                    int32_t* acc_out_or_null, void* workspace, size_t workspace_bytes, void* stream);

/* RoPE + KV-cache store operands of NPL_EPI_ROPE_KV (see npl_rope_store_kv). */
typedef struct npl_rope_kv {
  const void* cos_table; /* fp16 [max_position, head_dim]                       */
  const void* sin_table;
  int max_position;
  const int64_t* positions;     /* [M]                                        */
  const int32_t* slot_mapping;  /* [M], negative = padding                    */
  void* q_out;                  /* fp16 [M, heads, head_dim]                  */
  void* k_cache;                /* fp16 [num_blocks, block_size, kv_heads, D] */
  void* v_cache;
  int num_blocks;
  int block_size;
  int heads;
  int kv_heads;
  int head_dim;
} npl_rope_kv;

/*
 * npl_w8a8_linear with the layer math around a decode linear fused in.
 * Activations (x_mode):
 *   NPL_X_INT8         qa/lda/sa as npl_w8a8_linear.
 *   NPL_X_F16_ABSMAX   x_f16 [M, K] (row stride ldx) quantised per token with
 *                      scale = scale_from_absmax(x_absmax[m]) (float bits of
 *                      max |x[m, :]|, e.g. an NPL_EPI_SILU_MUL absmax_out);
 *                      the call zeroes x_absmax[0..M) after reading it.
 *                      Same result as npl_quant_rows on x_f16.
 *   NPL_X_F16_RMSNORM  x_f16 RMSNorm-ed with norm_weight/eps, then quantised:
 *                      the same arithmetic as npl_rmsnorm_quant.
 *   The fp16 modes take M <= 64 (decode batches).
 * Epilogues: those of npl_w8a8_linear, plus
 *   NPL_EPI_SILU_MUL with absmax_out: absmax_out[m] (float bits, zero before
 *                      the call) receives max over the row of |out[m, :]|.
 *                      With q_out / q_scale as well (M <= 64): once every CTA
 *                      has stored its outputs, the kernel quantises out per
 *                      token (npl_quant_rows' arithmetic) into q_out int8
 *                      [M, N/2] (row stride N/2, 8-byte aligned) and q_scale
 *                      fp32 [M], and leaves absmax_out zero again: the down
 *                      projection's input without a separate launch. Needs
 *                      ld_out % 8 == 0 and a 16-byte aligned out.
 *   NPL_EPI_ROPE_KV    N = (heads + 2 kv_heads) * head_dim (packed q | k | v,
 *                      head blocks multiples of 128 rows): q and k get RoPE
 *                      exactly as npl_rope_store_kv; q -> rope.q_out; k and v
 *                      -> the caches at slot_mapping (out is not written).
 * Workspace: npl_linear_workspace_bytes(M, N, K), as npl_w8a8_linear.
 * Replaces, for one decode step, lightweight_runner.py:239-245 + w8a8.py:
 * 106-115 (RMSNorm and activation quantisation before the QKV, gate/up and
 * LM-head linears), the down projection's activation quantisation, and
 * paged_attention.py:1286-1294 (rotary_fn + store_kvcache).
 */
typedef struct npl_linear_args {
  int x_mode;
  const int8_t* qa;
  int lda;
  const float* sa;
  const void* x_f16;
  int ldx;
  int32_t* x_absmax;
  const void* norm_weight;
  float eps;
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
  npl_rope_kv rope;
  int8_t* q_out;   /* NPL_EPI_SILU_MUL with absmax_out, M <= 64: out quantised per token (see below) */
  float* q_scale;
} npl_linear_args;

int npl_w8a8_linear_ex(const npl_linear_args* args, void* workspace, size_t workspace_bytes, void* stream);

/*
 * npl_w8a8_linear without a workspace argument, for callers that cannot
 * allocate device memory: a plugin inside a host engine that owns all device
 * memory and passes only input/output buffers, a binding from a language
 * without a CUDA allocator, or a loop that must not call cudaMalloc (it can
 * synchronise the device). This entry point has no counterpart in the
 * reference; it computes exactly what npl_w8a8_linear computes.
 * Its scratch is a fixed array inside the library (~5 MiB per device, held
 * until the process exits): M <= 64 tokens on devices with at most 160 SMs;
 * larger M is rejected with NPL_ERR_ARG. Every call shares that array: calls
 * that overlap on the GPU (other streams, other host threads) race and give
 * wrong results. Each call clears the part it uses on its stream first. A
 * call outside stream capture looks up the array's address on the current
 * device; a call during capture reuses the last one, so make the first call
 * on each device before any stream capture.
 */
int npl_w8a8_linear_noalloc(const int8_t* qa, int lda, const float* sa, const int8_t* qw, int ldw,
                            const float* sw, const float* bias_or_null, int M, int N, int K, int epilogue,
                            const void* residual_or_null, int ld_res, void* out, int ld_out, int out_dtype,
                            int32_t* acc_out_or_null, void* stream);

/*
 * store_kvcache (paged_attention.py:353-383): key/value fp16 [T, Hkv, D]
 * (token stride ld_tok) are written to cache slot slot_mapping[t] (block =
 * slot / block_size, offset = slot % block_size) of the caches
 * [num_blocks, block_size, Hkv, D]; negative slots are skipped.
 */
int npl_store_kv(const void* key, const void* value, int ld_tok, int T, int Hkv, int D,
                 const int32_t* slot_mapping, void* k_cache, void* v_cache, int num_blocks,
                 int block_size, void* stream);

/*
 * RoPE + store on the packed QKV projection output (paged_attention.py:
 * 1284-1294: rotary_fn(q, k, cos, sin) then store_kvcache): qkv fp16
 * [T, (H + 2*Hkv) * D] (row stride ld_qkv) holds q | k | v. With cos/sin the
 * fp16 tables [max_position, D] indexed by positions[t] (int64),
 *   rot(x) = fp16(fp16(x * cos) + fp16(rotate_half(x) * sin))
 * q_out [T, H, D] <- rot(q); rot(k) and v are stored as npl_store_kv does.
 */
int npl_rope_store_kv(const void* qkv, int ld_qkv, int T, int H, int Hkv, int D, const void* cos_table,
                      const void* sin_table, int max_position, const int64_t* positions,
                      const int32_t* slot_mapping, void* q_out, void* k_cache, void* v_cache,
                      int num_blocks, int block_size, void* stream);

/*
 * Decode-only paged attention (q_len = 1), paged_attention.py:872-1030:
 * q fp16 [B, H, D] contiguous; caches fp16 [num_blocks, block_size, Hkv, D];
 * block_tables int32 [B, bt_stride] (first max_blocks entries used);
 * context_lens int32 [B]. out fp16 [B, H, D]. Softmax in fp32 over the
 * context; a row with context_len 0 (padded bucket row) yields zeros.
 * With q_out/q_scale given, each row out[b] (H*D values) is also quantised
 * per token as npl_quant_rows does: q_out int8 [B, H*D], q_scale fp32 [B]
 * (the O projection's input, w8a8.py:106-115).
 * D is 64 or 128; block_size a multiple of 64, or 8, 16 or 32; B <= 1024 and
 * B * H * ceil(max_blocks * block_size / 256) <= 2^18. The workspace
 * (npl_decode_attention_workspace_bytes) must be zero-filled before its first
 * use; every call leaves its counters and flags zero again, so calls of any
 * shape may share it when they are ordered on one stream.
 */
size_t npl_decode_attention_workspace_bytes(int B, int H, int D, int max_blocks, int block_size);
int npl_paged_decode_attention(const void* q, int B, int H, int Hkv, int D, const void* k_cache,
                               const void* v_cache, int num_blocks, int block_size,
                               const int32_t* block_tables, int bt_stride, int max_blocks,
                               const int32_t* context_lens, float scale, void* out, int8_t* q_out_or_null,
                               float* q_scale_or_null, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Causal varlen attention of multi-token rows (prefill and suffix prefill)
 * over the paged pool: replaces paged_varlen_attention (paged_attention.py:
 * 1142-1207; Triton kernel :1037-1139). q fp16 [total_q, H, D] (token stride
 * ld_q elements, heads contiguous); sequence b owns rows
 * [q_offsets[b], q_offsets[b] + q_lens[b]) and the first context_lens[b]
 * slots of its block table; query j of it sits at absolute position
 * context_lens[b] - q_lens[b] + j and sees keys 0..that position. Scores are
 * fp32 dot products times `scale`; online softmax in fp32 with the
 * probabilities rounded to fp16 for the P.V product (tcgen05 kind::f16, fp32
 * accumulation). out fp16 [total_q, H, D] (token stride ld_out); rows of no
 * sequence are not written. max_q_len >= every q_lens[b] sizes the launch.
 * D is 64 or 128; block_size a multiple of 8. Bad table entries or offsets
 * skip the access and set NPL_DEV code 5 (npl_device_status). No workspace,
 * no allocation, no synchronisation (graph-capturable).
 */
int npl_paged_prefill_attention(const void* q, int ld_q, int total_q, int H, int Hkv, int D, const void* k_cache,
                                const void* v_cache, int num_blocks, int block_size, const int32_t* block_tables,
                                int bt_stride, int max_blocks, const int32_t* context_lens, const int32_t* q_lens,
                                const int32_t* q_offsets, int B, int max_q_len, float scale, void* out, int ld_out,
                                void* stream);

/*
 * Tensor-parallel exchanges over NVLink peer memory (one process per GPU).
 * They replace, for decode batches, the NCCL path of a row-parallel linear
 * (the tensor-parallel variant of the reference's O / down projections,
 * paged_attention.py:118-124 and lightweight_runner.py:320-383, 539-552):
 *   npl_row_absmax -> all-reduce(MAX) -> npl_quant_rows_absmax   by npl_tp_absmax_quant
 *   all-reduce(SUM) of int32 partials -> npl_dequant             by npl_tp_allreduce_dequant
 * with identical results. Each rank owns one zero-filled exchange buffer of
 * npl_tp_exchange_bytes(world, max_elems) bytes (256-byte aligned) and maps
 * every peer's with npl_ipc_handle / npl_ipc_open (CUDA IPC); npl_tp_peers
 * lists all ranks' buffers as mapped in the calling process (buffers[rank] =
 * its own). All ranks make the same sequence of calls with the same shapes;
 * each call pushes this rank's data into every peer's buffer, raises a
 * per-slice sequence number there and waits (bounded, ~1 s; on expiry
 * NPL_DEV code 6 in npl_device_status and the output is not written) for
 * every peer's. No host work per call: capturable in a CUDA graph.
 * No counterpart in the reference, which runs on one device.
 */
#define NPL_TP_MAX_RANKS 8
#define NPL_IPC_HANDLE_BYTES 64
typedef struct {
  int world;
  int rank;
  void* buffers[NPL_TP_MAX_RANKS];
  long long max_elems; /* the largest M * N of npl_tp_allreduce_dequant (multiple of 4) */
} npl_tp_peers;

size_t npl_tp_exchange_bytes(int world, long long max_elems);
/* CUDA IPC of a device buffer: the handle (NPL_IPC_HANDLE_BYTES) of the
 * allocation holding `ptr` and the offset of `ptr` in it; npl_ipc_open maps a
 * peer's handle into this process (ptr_out = base_out + offset);
 * npl_ipc_close unmaps base_out. */
int npl_ipc_handle(const void* ptr, void* handle_out, size_t* offset_out);
int npl_ipc_open(const void* handle, size_t offset, void** ptr_out, void** base_out);
int npl_ipc_close(void* base);
/* x fp16 [M, K] (this rank's columns of each row, row stride ldx), M <= 64:
 * q int8 [M, K] (row stride ldq) and scale[M] as npl_quant_rows would give
 * for the whole rows spread over the ranks (the scale from the max over all
 * ranks' absmax). K % 16 == 0. */
int npl_tp_absmax_quant(const npl_tp_peers* peers, const void* x, int M, int K, int ldx, int8_t* q, int ldq,
                        float* scale, void* stream);
/* acc int32 [M, N] contiguous: this rank's partial accumulators. out fp16
 * [M, N] = npl_dequant of the sum over all ranks' acc (NPL_EPI_RESIDUAL when
 * residual is given, else NPL_EPI_NONE). N % 4 == 0, M * N <= max_elems. */
int npl_tp_allreduce_dequant(const npl_tp_peers* peers, const int32_t* acc, int M, int N, const float* sa,
                             const float* sw, const float* bias_or_null, const void* residual_or_null, int ld_res,
                             void* out, int ld_out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NPL_W8A8_H_ */
