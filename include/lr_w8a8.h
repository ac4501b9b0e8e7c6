/*
 * lr_w8a8.h — C ABI of the B200 (sm_100a) W8A8 projection path of
 * LynnReal-Omni Flash DiT blocks.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a cudaStream_t passed as void*;
 *   - launches asynchronously on that stream and never synchronises;
 *   - allocates nothing: outputs are caller-owned buffers;
 *   - returns LR_OK or an error status; lr_last_error() then holds a message.
 *
 * Tensor conventions (all row-major, C-contiguous unless a stride is given):
 *   bf16 values are passed as `const void*` / `void*` (2 bytes per element);
 *   `indices` are int64 adaLN table rows, one per token of the sequence: the
 *   table row of flattened row r is indices[r % sequence]
 *   (model/kernels.py:62-63,98-99,144-145);
 *   `table` is the bf16 adaLN modulation table [table_rows, table_width] with
 *   slot s occupying columns [s*hidden, (s+1)*hidden) (model/fusion.py:69).
 *
 * Numerics follow model/kernels.py and model/int8_gemm.py with IEEE
 * division / square root and no FMA contraction; the rounding points are
 * documented per function.
 */
#ifndef LR_W8A8_H
#define LR_W8A8_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define LR_OK 0
#define LR_ERR_INVALID_ARGUMENT 1 /* contract violation (reference raises ValueError) */
#define LR_ERR_UNSUPPORTED 2      /* shape or alignment this build does not handle */
#define LR_ERR_CUDA 3             /* a CUDA runtime/driver call failed */

/* GEMM epilogues (lr_int8_gemm). */
#define LR_EPI_NONE 0          /* bf16((acc*rs)*cs + bias) */
#define LR_EPI_GELU_TANH 1     /* bf16(gelu_tanh(bf16((acc*rs)*cs + bias))) */
#define LR_EPI_GATED_RESIDUAL 2 /* bf16(x + bf16(gate * bf16((acc*rs)*cs + bias))) */

/* Library version (major*10000 + minor*100 + patch). */
int lr_version(void);

/* Message describing the last error returned on this host thread ("" if none). */
const char* lr_last_error(void);

/* Read (and, if clear != 0, reset) the device status bits of the current device.
 * Bit 0: an adaLN index was outside [0, table_rows) (that row used a zero
 * modulation); bit 1: a bounded wait inside the GEMM gave up; bit 2: a row
 * index of lr_gather_rows / lr_flash_restore was outside its source (that
 * output row was written from zeros). Bit 1 also covers the attention
 * kernel's bounded waits. Synchronises the device. */
int lr_device_status(unsigned int* bits, int clear);

/* Arithmetic of the divisions and RMS reciprocal square roots of the
 * element-wise kernels (K1, K3, K4, K7, K8 and the Q/K RMSNorm) on the current
 * device:
 *   LR_ARITH_REFERENCE_GPU (default): as the reference's Triton kernels
 *     compile on the GPU (model/kernels.py:13-14, 65, 106, 121-126: fp32 `/`
 *     is div.full.f32, tl.rsqrt is rsqrt.approx.f32), so the int8
 *     activations and row scales equal what the reference computes on the
 *     same GPU;
 *   LR_ARITH_IEEE: IEEE round-to-nearest division and square root, as the
 *     reference's PyTorch path (model/int8.py:66-67) and its kernels under
 *     the Triton interpreter compute them; a CPU restatement reproduces it.
 * Sums of squares use one order in both modes: the reference's compiled
 * tl.sum order (8 warps, 8 columns per thread; exact for rows of 2048 or more
 * columns). Set it before launching work on the device. */
#define LR_ARITH_IEEE 0
#define LR_ARITH_REFERENCE_GPU 1
/* LR_ARITH_TORCH_CUDA (lr_quantize_rows_arith only): the reference's unfused
 * PyTorch quantiser as it runs on a CUDA device (Int8Linear.forward with
 * fused_ops off, model/int8.py:66-67). PyTorch divides a CUDA tensor by a
 * scalar as a multiply by the float reciprocal, so
 *   scale = fl(max(absmax, 1e-8) * fl(1/127)),  q = RNE(clamp(x / scale)) (IEEE /). */
#define LR_ARITH_TORCH_CUDA 2
int lr_set_arithmetic(int mode);
int lr_get_arithmetic(int* mode);

/* K1 — per-row dynamic int8 quantisation.
 * Replaces model/kernels.py:19-24 `quantize_rows` (kernel :8-16) and the torch
 * quantiser of Int8Linear.forward, model/int8.py:66-67.
 *   scale[r] = max(max_j |x[r,j]|, 1e-8) / 127        (fp32)
 *   q[r,j]   = round_half_even(clamp(x[r,j] / scale[r], -127, 127))
 * x: bf16 [rows, width] with row stride `row_stride` elements (>= width);
 * q: int8 [rows, width] contiguous; scales: fp32 [rows]. */
int lr_quantize_rows(const void* x, int64_t rows, int64_t width, int64_t row_stride,
                     int8_t* q, float* scales, void* stream);

/* K1 with the arithmetic chosen per call instead of the device's mode:
 * LR_ARITH_IEEE, LR_ARITH_REFERENCE_GPU or LR_ARITH_TORCH_CUDA. Int8Linear's
 * unfused quantiser (model/int8.py:66-67) runs as LR_ARITH_TORCH_CUDA. */
int lr_quantize_rows_arith(const void* x, int64_t rows, int64_t width, int64_t row_stride,
                           int8_t* q, float* scales, int arithmetic, void* stream);

/* K2 — standalone int32 -> bf16 dequant epilogue.
 * Replaces model/kernels.py:41-46 `int8_epilogue` (kernel :27-38), used by
 * Int8Linear.forward_quantized with gemm="torch" and fused_ops (model/int8.py:52-54).
 *   out[m,n] = bf16((float(acc[m,n]) * row_scale[m]) * col_scale[n] + bias[n])
 * bias may be NULL. */
int lr_int8_epilogue(const int32_t* acc, int64_t rows, int64_t cols, const float* row_scale,
                     const float* col_scale, const void* bias, void* out, void* stream);

/* K3 — RMSNorm + adaLN modulate, bf16 output.
 * Replaces model/kernels.py:260-272 `_rms_adaln` (kernel :48-78).
 *   r   = 1 / sqrt(sum_j x^2 / hidden + eps)
 *   n   = bf16((x * r) * w)
 *   out = bf16(bf16(n * bf16(1 + table[.., scale_slot])) + table[.., shift_slot])
 * x, out: bf16 [rows, hidden]; norm_weight: bf16 [hidden]. */
int lr_rms_adaln(const void* x, const void* norm_weight, float eps, const void* table,
                 int64_t table_rows, int64_t table_width, const int64_t* indices, int64_t sequence,
                 int64_t rows, int64_t hidden, int shift_slot, int scale_slot, void* out,
                 void* stream);

/* K4 (+K8) — RMSNorm + adaLN modulate + per-row int8 quantisation.
 * Replaces model/kernels.py:275-289 `_rms_adaln_quant_int8` (kernel :81-128)
 * and, when `update` is non-NULL, model/kernels.py:405-419 `residual_rms_quant`
 * (the kernel's WITH_RESIDUAL branch, :101-105):
 *   v = x;  if update: v = bf16(x + bf16(table[.., gate_slot] * update)),
 *                      residual_out = v
 *   m = bf16(bf16(n * bf16(1 + scale)) + shift) with n as in lr_rms_adaln
 *   scales[r] = max(max_j |m|, 1e-8) / 127; q = RNE(clamp(m / scales[r], +-127))
 * table may be NULL: then no modulation is applied (m = n) and the gate is 1
 * (a plain RMSNorm + quantiser, used for slot-free prologues). */
int lr_rms_adaln_quant_int8(const void* x, const void* norm_weight, float eps, const void* table,
                            int64_t table_rows, int64_t table_width, const int64_t* indices,
                            int64_t sequence, int64_t rows, int64_t hidden, int shift_slot,
                            int scale_slot, const void* update, int gate_slot, void* residual_out,
                            int8_t* q, float* scales, void* stream);

/* K5 — gated residual.
 * Replaces model/kernels.py:292-304 `_gated_residual` (kernel :131-153):
 *   out = bf16(x + bf16(table[indices[r % sequence], gate_slot*hidden + j] * y))
 * table may be NULL (gate = 1: a plain bf16 residual add). */
int lr_gated_residual(const void* x, const void* y, const void* table, int64_t table_rows,
                      int64_t table_width, const int64_t* indices, int64_t sequence, int64_t rows,
                      int64_t hidden, int gate_slot, void* out, void* stream);

/* K6 — SwiGLU on a [rows, 2*inner] projection (value | gate halves).
 * Replaces model/kernels.py:307-315 `_swiglu` (kernel :156-166):
 *   out = bf16(value * bf16(gate * sigmoid(gate))) */
int lr_swiglu(const void* projected, int64_t rows, int64_t inner, void* out, void* stream);

/* K7 — SwiGLU + per-row int8 quantisation.
 * Replaces model/kernels.py:318-328 `_swiglu_quant_int8` (kernel :169-185). */
int lr_swiglu_quant_int8(const void* projected, int64_t rows, int64_t inner, int8_t* q,
                         float* scales, void* stream);

/* K9 — per-head RMSNorm + rotary embedding of Q and K (the step after the QKV
 * projection). Replaces the reference's `_qk_norm_full_rope_paired_kernel`
 * (model/kernels.py:188-257) and `_qk_norm_rope_kernel` (:345-402) as launched
 * by FusedAttention (model/fusion.py:29-54). For each (batch b, token t,
 * head h) row of Q (and likewise K):
 *   r = 1 / sqrt(sum_d x^2 / head_dim + eps);  n = bf16((x * r) * w)
 *   d <  rotary_dim: out = bf16(bf16(n_d * c) + bf16(+-n_pair * s)),
 *        c, s = bf16(cos[t, d]), bf16(sin[t, d]), pair = d -+ rotary_dim/2
 *        (minus sign for the first half)
 *   d >= rotary_dim: out = n_d
 * query/key rows start at b*sequence*token_stride + t*token_stride +
 * h*head_stride (bf16, unit element stride); cos/sin: fp32 [sequence,
 * rotary_dim]; q_out/k_out: bf16 [batch, sequence, heads, head_dim] contiguous.
 * head_dim <= 256, rotary_dim even and <= head_dim. */
int lr_qk_norm_rope(const void* query, const void* key, int64_t q_token_stride,
                    int64_t q_head_stride, int64_t k_token_stride, int64_t k_head_stride,
                    const void* q_weight, const void* k_weight, const float* cos, const float* sin,
                    int64_t batch, int64_t sequence, int64_t heads, int64_t head_dim,
                    int64_t rotary_dim, float eps, void* q_out, void* k_out, void* stream);

/* F1 — row gather (the index_select calls of Flash token compression).
 * Replaces the Tensor.index_select calls of model/flash.py:71-79 (hidden rows
 * along the sequence, adaLN indices, rotary rows, attention-mask columns):
 *   out[o, i, :] = src[o, index[i], :]   for o < outer, i < n_index,
 * where a "row" is `row_bytes` contiguous bytes, src slice o starts at byte
 * o * src_outer_stride and out slice o at byte o * out_outer_stride. Any
 * element type: the copy is bytewise (16-byte vectors when sizes and pointers
 * allow). An index outside [0, src_rows) sets status bit 2 and writes zeros. */
int lr_gather_rows(const void* src, int64_t outer, int64_t src_outer_stride, int64_t src_rows,
                   int64_t row_bytes, const int64_t* index, int64_t n_index, void* out,
                   int64_t out_outer_stride, void* stream);

/* F2 — Flash residual restore before the first full-resolution suffix block.
 * Replaces the `restore` hook of model/flash.py:81-84 (a subtract, a scale,
 * an index_select and an add over four tensors) with one pass:
 *   k = inverse[t]
 *   out[b,t,:] = bf16(full[b,t,:] + bf16(bf16(compressed[b,k,:] - input[b,k,:]) * gain))
 * full, out: bf16 [batch, sequence, hidden]; compressed (the last compressed
 * block's output) and input (the compressed sequence that entered the first
 * compressed block): bf16 [batch, kept, hidden]; inverse: int64 [sequence].
 * out may alias full. */
int lr_flash_restore(const void* full, const void* compressed, const void* input,
                     const int64_t* inverse, int64_t batch, int64_t sequence, int64_t kept,
                     int64_t hidden, float gain, void* out, void* stream);

/* F3 — nearest same-time anchor of every dropped video row (the cdist/argmin
 * loop of spatial_layout, model/flash.py:27-32):
 *   for r < n_dropped: src = dropped[r];
 *     best = argmin over j with positions[anchors[j],0] == positions[src,0] of
 *            |positions[src,1:3] - positions[anchors[j],1:3]|  (first j on ties;
 *            0 if no anchor shares the time);
 *     inverse[src] = inverse[anchors[best]]
 * positions: fp32 [sequence, 3] (time, row, column); the distance is the fp32
 * square root of the squared distance, which equals the reference's fp32
 * cdist wherever that is exact (integer coordinates below 2^11). */
int lr_flash_nearest_anchor(const float* positions, int64_t sequence, const int64_t* dropped,
                            int64_t n_dropped, const int64_t* anchors, int64_t n_anchors,
                            int64_t* inverse, void* stream);

/* A1 — attention core (bf16): for every batch b, query i, head h
 *   out[b,i,h,:] = sum_j softmax_j(scale * q[b,i,h,:] . k[b,j,h,:]) * v[b,j,h,:]
 * with fp32 scores and an fp32 online softmax (exp2), probabilities rounded to
 * bf16 for the second product, bf16 output. Stands in for the attention
 * backend FusedAttention calls between the Q/K RMSNorm+RoPE and the output
 * projection (model/fusion.py:55-57; the reference calls diffusers'
 * dispatch_attention_fn, i.e. a library SDPA kernel). No mask, not causal.
 * q, k, v, out: bf16 [batch, seq, heads, head_dim] with heads contiguous inside
 * a token and token strides in elements (a fused QKV output's views work
 * as they are); head_dim must be 128; pointers and token strides 16-byte
 * aligned (LR_ERR_UNSUPPORTED otherwise). */
int lr_attention_bf16(const void* q, int64_t q_token_stride, const void* k, int64_t k_token_stride,
                      const void* v, int64_t v_token_stride, int64_t batch, int64_t seq_q, int64_t seq_kv,
                      int64_t heads, int64_t head_dim, float scale, void* out, int64_t out_token_stride,
                      void* stream);

/* K10 (+K2 fused) — INT8 GEMM with int32 accumulation and a fused bf16 epilogue.
 * Replaces model/int8_gemm.py:96-163 `int8_matmul` (kernel `_gemm` :13-46),
 * model/int8_tma.py:32-41 `matmul`, and the GEMM inside
 * Int8Linear.forward_quantized (model/int8.py:41-58).
 *   acc[m,n] = sum_k a[m,k] * b[k,n]                       (exact int32)
 *   d[m,n]   = (float(acc) * row_scale[m]) * col_scale[n] (+ bias[n])
 * a: int8 [M, K], row stride lda (elements, >= K);
 * b: int8 weights addressed as b[k*b_stride_k + n*b_stride_n] — the
 *    reference's `weight_int8` is the [K, N] transpose view of a row-major
 *    [N, K] matrix, i.e. b_stride_k = 1, b_stride_n = K (model/int8.py:12,33);
 * row_scale: fp32 [M]; col_scale: fp32 [N]; bias: bf16 [N] or NULL;
 * out: bf16 [M, N] row stride ldo.
 * epilogue LR_EPI_GATED_RESIDUAL additionally reads the residual stream
 * `resid` (bf16 [M, N], row stride ldr; may alias `out` only if ldr == ldo)
 * and the gate table[indices[m % sequence], gate_slot*N + n]; `table` may be
 * NULL for gate = 1 (plain residual add). Unused residual arguments may be 0/NULL.
 * The tensor-core path (tcgen05, TMA) needs b_stride_k == 1, lda % 16 == 0,
 * b_stride_n % 16 == 0, 16-byte aligned a/b/out and N, ldo (and ldr) multiples
 * of 8; other layouts
 * run a CUDA-core kernel with identical results. */
int lr_int8_gemm(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                 int64_t b_stride_n, int64_t M, int64_t N, int64_t K, const float* row_scale,
                 const float* col_scale, const void* bias, int epilogue, const void* resid,
                 int64_t ldr, const void* table, int64_t table_rows, int64_t table_width,
                 const int64_t* indices, int64_t sequence, int gate_slot, void* out, int64_t ldo,
                 void* stream);

/* Bytes of int32 workspace lr_int8_gemm_ws uses for this shape (slices x M x N
 * int32), or 0 when the shape has enough output tiles to fill the GPU without
 * splitting K. */
int64_t lr_int8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* lr_int8_gemm with a caller-provided device workspace (no counterpart in the
 * reference, which has no split-K). For shapes whose output tiles cannot fill
 * the GPU (small M), K is split across CTA pairs: every K slice stores its
 * partial int32 accumulators into its own M x N plane of the workspace, and a
 * second kernel adds the planes in slice order (exact integer adds) and applies
 * the epilogue. Results are identical to lr_int8_gemm. With workspace == NULL, or
 * workspace_bytes < lr_int8_gemm_workspace_bytes(M, N, K), or a shape that
 * needs no split, it behaves exactly like lr_int8_gemm. Calls sharing one
 * workspace must be ordered on one stream. */
int lr_int8_gemm_ws(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                    int64_t b_stride_n, int64_t M, int64_t N, int64_t K, const float* row_scale,
                    const float* col_scale, const void* bias, int epilogue, const void* resid,
                    int64_t ldr, const void* table, int64_t table_rows, int64_t table_width,
                    const int64_t* indices, int64_t sequence, int gate_slot, void* out,
                    int64_t ldo, void* workspace, int64_t workspace_bytes, void* stream);

/* lr_int8_gemm whose output rows go to several places at once: the row m of
 * the result is written to row row_offset + m of each of the
 * `num_destinations` (1 to 8) bf16 matrices `destinations[d]` (leading
 * dimension ld_destination), which may be other GPUs' memory mapped into this
 * process (lr_ipc_import). No counterpart in the reference, which gathers
 * sharded rows, if at all, with a separate collective: here the GEMM epilogue
 * is the all-gather, its bulk tensor stores to every rank's copy of the
 * gathered tensor overlapping the tensor-core work over NVLink. The kernel
 * returns only once every store has landed; making the writes visible to the
 * other GPUs' next kernels takes a cross-GPU barrier after it (an NCCL
 * collective on the same stream), and no GPU may read or write the
 * destination rows while the call runs. Needs the CTA-pair tensor-core path
 * (K-major 16-byte aligned operands, M > 128), N a multiple of 32,
 * ld_destination a multiple of 8 and 16-byte aligned destinations; otherwise
 * LR_ERR_UNSUPPORTED. Epilogues and results as lr_int8_gemm (`out` is the
 * destinations). */
int lr_int8_gemm_rows_to(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                         int64_t b_stride_n, int64_t M, int64_t N, int64_t K, const float* row_scale,
                         const float* col_scale, const void* bias, int epilogue, const void* resid,
                         int64_t ldr, const void* table, int64_t table_rows, int64_t table_width,
                         const int64_t* indices, int64_t sequence, int gate_slot,
                         void* const* destinations, int num_destinations, int64_t ld_destination,
                         int64_t row_offset, void* stream);

/* CUDA IPC of device buffers between the processes of one node (one process
 * per GPU), for lr_int8_gemm_rows_to's peer destinations. No counterpart in
 * the reference (it has no multi-GPU code). lr_ipc_export writes the 64-byte
 * handle of the cudaMalloc allocation holding `ptr` and ptr's offset in it;
 * lr_ipc_import maps such a handle from another process on the current device
 * and returns the pointer at `offset` (peer access enabled lazily);
 * lr_ipc_release unmaps it. The exporting process must keep the buffer alive
 * while others map it. */
#define LR_IPC_HANDLE_BYTES 64
int lr_ipc_export(const void* ptr, void* handle, int64_t* offset);
int lr_ipc_import(const void* handle, int64_t offset, void** ptr);
int lr_ipc_release(void* ptr, int64_t offset);

/* Test hook of the GEMM's bounded waits (no counterpart in the reference):
 * sets, on the current device, the limit of every mbarrier wait of the
 * tensor-core GEMM kernels (limit_ns; 0 restores the default of 2 s) and,
 * with drop_first_load != 0, makes the next launch of the CTA-pair kernel
 * skip one TMA load of its first stage, so that stage's barrier never
 * completes. That launch's waits then run out: the kernel raises device status
 * bit 1, drains its own copies and tensor-core work, frees its tensor memory
 * and returns after a few limits; its output is unspecified. Later launches
 * are unaffected. Not for production use. */
int lr_gemm_test_wait(int64_t limit_ns, int drop_first_load);

/* Size of the fixed split-K scratch array behind lr_int8_gemm_noalloc. */
#define LR_NOALLOC_SCRATCH_BYTES (16ll << 20)

/* lr_int8_gemm for callers that cannot allocate device memory — a plugin or
 * FFI host that only hands over the tensors it already owns, or a framework
 * whose memory pool must not grow during a step. No counterpart in the
 * reference. Same arguments and same results as lr_int8_gemm; where the shape
 * is small enough in M to split K (lr_int8_gemm_workspace_bytes > 0), the
 * split-K scratch is a fixed 16 MiB array compiled into this library, which
 * every GPU that loads the library holds until the process exits. It calls no
 * cudaMalloc or cudaFree and never allocates.
 *   - A shape whose split-K scratch exceeds LR_NOALLOC_SCRATCH_BYTES is
 *     rejected with LR_ERR_UNSUPPORTED (use lr_int8_gemm_ws with a workspace).
 *   - The first call on each device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture. Under CUDA's lazy module loading (the
 *     default) that first call, or the library's first kernel launch on the
 *     device, is also when the GPU code is loaded and the 16 MiB array
 *     allocated: make it at set-up time, not inside a step whose memory must
 *     not grow. Later calls allocate nothing.
 *   - All calls share the one array and it keeps the last call's contents;
 *     nothing in it needs to start at zero (each call writes every element it
 *     later reads). Calls that overlap on the GPU (concurrent streams, or
 *     several host threads) race on the array: order them on one stream. */
int lr_int8_gemm_noalloc(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                         int64_t b_stride_n, int64_t M, int64_t N, int64_t K,
                         const float* row_scale, const float* col_scale, const void* bias,
                         int epilogue, const void* resid, int64_t ldr, const void* table,
                         int64_t table_rows, int64_t table_width, const int64_t* indices,
                         int64_t sequence, int gate_slot, void* out, int64_t ldo, void* stream);

/* Raw int32 accumulators of the same GEMM (exactness checks of the integer path):
 *   acc[m,n] = sum_k a[m,k] * b[k,n], acc row stride N. */
int lr_int8_gemm_s32(const int8_t* a, int64_t lda, const int8_t* b, int64_t b_stride_k,
                     int64_t b_stride_n, int64_t M, int64_t N, int64_t K, int32_t* acc,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LR_W8A8_H */
