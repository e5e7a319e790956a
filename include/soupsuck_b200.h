/* soupsuck_b200: C ABI of the B200 (sm_100a) QLoRA hot path.
 *
 * Every entry point takes raw device pointers, element counts and strides, and
 * a CUDA stream passed as `void*` (a cudaStream_t; NULL = legacy default
 * stream).  Nothing here allocates device memory: callers pass outputs and, where
 * a routine needs scratch space, a workspace whose size the matching
 * `*_workspace_bytes` query reports.  Every function returns 0 on success or one
 * of the SB_E* codes; `sb_last_error()` then describes the failure (per thread).
 * Invalid arguments are rejected before any launch.  No kernel traps the GPU:
 * a device-side wait that runs out (bounded spin loops) records an error code
 * that `sb_take_device_error()` reports.
 *
 * 16-bit floating-point buffers are IEEE binary16 passed as `uint16_t*`.
 * Where a routine accepts either binary16 or binary32, a dtype code selects it.
 *
 * Reference interface citations are paths inside the Khasuetolog/soupsuck
 * project; each entry point replaces the Triton launch (or library GEMM) named
 * beside it.
 */
#ifndef SOUPSUCK_B200_H
#define SOUPSUCK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  SB_OK = 0,
  SB_EINVAL = 1,       /* unsupported shape, dtype, alignment or NULL pointer */
  SB_ECUDA = 2,        /* a CUDA runtime call failed */
  SB_EUNSUPPORTED = 3, /* no kernel for this case on this device */
  SB_EWORKSPACE = 4    /* workspace smaller than the *_workspace_bytes query */
};

enum { SB_F16 = 0, SB_F32 = 1 };

/* Library identity and error reporting. */
int sb_abi_version(void);
const char* sb_last_error(void);
/* Reads and clears the device-side error word (bounded-wait timeouts inside the
 * tcgen05 kernels).  *flag = 0 means no kernel gave up waiting since the last call.
 * Synchronises `stream`. */
int sb_take_device_error(void* stream, int* flag);
/* Number of kernels this library launched since load (a process-wide counter). */
int64_t sb_launch_count(void);

/* ---------------------------------------------------------------- NF4 decode
 * Replaces nf4_decode_kernel (solution/kernels/nf4.py:41-59) as launched by
 * dequantize_nf4 (:190-203, NESTED=True) and _dequantize_flat_into (:181-187,
 * NESTED=False).  out[i] = fp16_rn(NF4[nib(i)] * scale(i // 64)); bit-exact. */
int sb_nf4_dequant_nested(const uint8_t* packed, const uint8_t* qabs, const float* absmax2,
                          const float* code2, const float* offset, uint16_t* out, int64_t n,
                          void* stream);
int sb_nf4_dequant_flat(const uint8_t* packed, const float* absmax, uint16_t* out, int64_t n,
                        void* stream);

/* ---------------------------------------------------------------- NF4 linear
 * A bitsandbytes nested NF4 weight W[n_out, k_in] (row-major element order,
 * QuantState.shape = (n_out, k_in)), as validated by _validate_state
 * (solution/kernels/nf4.py:140-168). */
typedef struct {
  const uint8_t* packed;  /* ceil(n_out*k_in/2) bytes, high nibble = earlier element */
  const uint8_t* qabs;    /* ceil(n_out*k_in/64) uint8 codes into code2 */
  const float* absmax2;   /* one fp32 scale per 256 blocks */
  const float* code2;     /* 256 fp32 code values */
  const float* offset;    /* one fp32 value */
  int64_t n_out;
  int64_t k_in;
} sb_nf4_weight;

/* Forward: Y[m, n_out] = X[m, k_in] . deq(W)^T + lora_a[m, r] . lora_b[n_out, r]^T + bias.
 * Replaces the base projection (bnb MatMul4Bit -> F.linear, mirrored by
 * nf4_tile_matmul_kernel TRANSPOSE=False, solution/kernels/nf4_gemm.py:35-71)
 * plus the LoRA up-projection and lora_scale_add_kernel
 * (solution/kernels/lora_epilogue.py:24-34) of the patched PEFT forward
 * (solution/lora.py:135-164).  lora_a is the already-scaled s*(X.A^T) in fp16
 * (sb_lora_project); pass lora_a = lora_b = NULL, r = 0 for a frozen projection.
 * X, Y, bias, lora_* are fp16, fp32 accumulation. */
int sb_nf4_linear_fwd(const uint16_t* x, int64_t m, const sb_nf4_weight* w,
                      const uint16_t* bias, const uint16_t* lora_a, const uint16_t* lora_b,
                      int r, uint16_t* y, void* workspace, size_t workspace_bytes, void* stream);

/* Backward input gradient: dX[m, k_in] = dY[m, n_out] . deq(W) + lora_a[m, r] . lora_b[k_in, r]^T.
 * Replaces MatMul4Bit.backward's dequantize + torch.matmul
 * (solution/nf4_patch.py:62-87, mirrored at solution/kernels/nf4_gemm.py:109-118,
 * TRANSPOSE=True) plus the LoRA dX term.  lora_a = s*(dY.B) in fp16
 * (sb_lora_project), lora_b = A^T laid out [k_in, r] (sb_lora_prepare). */
int sb_nf4_linear_dx(const uint16_t* dy, int64_t m, const sb_nf4_weight* w,
                     const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* dx,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes the two calls above need for these sizes, assuming 16-byte aligned
 * x/dy, packed and LoRA pointers: fp32 partial tiles and per-tile counters when the
 * tcgen05 path splits tiles across CTAs (stream-K), the fp32 reduction-slice
 * partials of the decode-to-shared small-M kernel (m <= 16 with SB_SMALLM=mma; the
 * default small-M kernels reduce through cluster shared memory and need none), or
 * the decoded weight when an odd shape takes the CUDA-core path. */
size_t sb_nf4_linear_workspace_bytes(int64_t m, int64_t n_out, int64_t k_in, int dx);

/* ---------------------------------------------------------------- LoRA factors
 * The low-rank products around the base projection: the PEFT lora_A / lora_B
 * nn.Linear pair under fp16 autocast (solution/lora.py:161) and its autograd
 * backward.  Rank r is 16, 32 or 64 (smaller ranks are zero-padded by the caller).
 *
 * sb_lora_prepare: lora_A [r, k] and lora_B [n, r] (fp16 or fp32) -> fp16 copies
 *   a16 [r, k], at16 [k, r], b16 [n, r], bt16 [r, n] (any output may be NULL).
 * sb_lora_project: P = X[m, k] . W[r, k]^T; writes fp16(scale_rows * P) row-major
 *   with row pitch ld_rows, and/or fp16(scale_t * P)^T as [r, ldt] with rows
 *   m..ldt-1 of the last 16-row tile zero-filled.  k % 32 == 0, 16-byte aligned
 *   x and w.  Forward: Z = X.A^T (W = a16); backward: U = dY.B (W = bt16).
 * sb_lora_reduce: out[r, w] = scale * Pt[r, ldp] . Q[ldp, w] over the first m rows
 *   of Q (rows m..ldp-1 of Pt must be zero), out transposed to [w, r] when
 *   transpose != 0, stored in out_dtype.  dA = U^T.X; dB = s * (Z^T.dY)^T.
 *   Deterministic two-stage reduction through `workspace`
 *   (sb_lora_reduce_workspace_bytes(m, w, r) bytes). */
int sb_lora_prepare(const void* a, int a_dtype, const void* b, int b_dtype, int r, int64_t k,
                    int64_t n, uint16_t* a16, uint16_t* at16, uint16_t* b16, uint16_t* bt16,
                    void* stream);
/* sb_lora_prepare_pair: two adapters of one input (gate and up) as one rank-2r adapter:
 *   a1, a2 [r, k] and b1, b2 [n, r] -> fp16 a_cat [2r, k] (a1 over a2), at_cat [k, 2r],
 *   b_bd [2n, 2r] = [[b1, 0], [0, b2]] and bt_bd [2r, 2n].  No counterpart in the
 *   reference, whose gate/up projections carry no adapters together. */
int sb_lora_prepare_pair(const void* a1, const void* a2, int a_dtype, const void* b1, const void* b2,
                         int b_dtype, int r, int64_t k, int64_t n, uint16_t* a_cat, uint16_t* at_cat,
                         uint16_t* b_bd, uint16_t* bt_bd, void* stream);
int sb_lora_project(const uint16_t* x, int64_t m, int64_t k, const uint16_t* w, int r,
                    float scale_rows, uint16_t* out_rows, int ld_rows, float scale_t,
                    uint16_t* out_t, int64_t ldt, void* stream);
size_t sb_lora_reduce_workspace_bytes(int64_t m, int64_t w, int r);
int sb_lora_reduce(const uint16_t* pt, int64_t ldp, const uint16_t* q, int64_t m, int64_t w, int r,
                   float scale, int transpose, void* out, int out_dtype, void* workspace,
                   size_t workspace_bytes, void* stream);
/* sb_lora_dual: the two products of the LoRA backward that read the upstream
 * gradient Q = dY [m, w] (16-byte aligned, w % 8 == 0), from one pass over it:
 *   dB = scale_b * Pt . Q  (Pt = Z^T [r, ldp], rows m..ldp-1 zero), [r, w] or
 *        transposed [w, r], in db_dtype -- the sb_lora_reduce of dB;
 *   U  = Q . Bt^T          (Bt [r, w]), fp16(scale_rows * U) row-major with pitch
 *        ld_rows and/or fp16(scale_t * U)^T [r, ldt] (ldt = m rounded up to 16,
 *        rows m..ldt-1 zero) -- the sb_lora_project of U.
 * wsplit = 0: dense, r = 16 or 32.  wsplit > 0 (a multiple of 256): two adapters
 * side by side (the gate/up pair, r = 32 or 64): columns below wsplit pair with
 * factor rows [0, r/2), the others with [r/2, r); U is the full product (Bt's
 * off-diagonal blocks are zero) and dB only its diagonal blocks, [r/2, w] (or
 * [w, r/2]) with each column's rows counted from its block's first.
 * pt = NULL: U only (db_out unused) -- the forward's Z = X.A^T for long rows.
 * Deterministic; workspace sb_lora_dual_workspace_bytes(m, w, r, wsplit).
 * Replaces the projection + reduction pair of the LoRA backward
 * (solution/lora.py:161 under autograd: lora_B's weight gradient and input
 * gradient read the same upstream gradient). */
size_t sb_lora_dual_workspace_bytes(int64_t m, int64_t w, int r, int64_t wsplit);
int sb_lora_dual(const uint16_t* q, int64_t m, int64_t w, const uint16_t* pt, int64_t ldp, const uint16_t* bt,
                 int r, int64_t wsplit, float scale_b, int transpose_b, void* db_out, int db_dtype,
                 float scale_rows, uint16_t* u_rows, int ld_rows, float scale_t, uint16_t* u_t, int64_t ldt,
                 void* workspace, size_t workspace_bytes, void* stream);
/* sb_lora_reduce without any allocation or workspace, for callers that cannot
 * allocate device memory (memory planned once at start-up, foreign-language
 * bindings without a CUDA allocator, steps that must not grow their footprint).
 * No counterpart in the reference: its reduction always allocates through the
 * PyTorch caching allocator.  The fp32 partial sums live in one fixed 8 MiB
 * device array inside this library (kept by every GPU that loads it until the
 * process exits); r * w above 2,097,152 is rejected with SB_EINVAL.  All calls
 * share that array and calls that overlap on the GPU race on it; nothing in it
 * has to start at zero.  The first call on a device looks up the array with
 * that device current: make it before any stream capture. */
int sb_lora_reduce_static(const uint16_t* pt, int64_t ldp, const uint16_t* q, int64_t m, int64_t w,
                          int r, float scale, int transpose, void* out, int out_dtype, void* stream);

/* ---------------------------------------------------------------- LoRA epilogue
 * lora_scale_add_kernel / lora_scale_gradient_kernel
 * (solution/kernels/lora_epilogue.py:24-43), elementwise, bit-exact. */
int sb_lora_scale_add(const void* base, int base_dtype, const void* adapter, int adapter_dtype,
                      void* out, int out_dtype, int64_t count, float scale, int cast_to_base,
                      void* stream);
int sb_lora_scale_grad(const void* grad, int grad_dtype, void* dadapter, int adapter_dtype,
                       int64_t count, float scale, void* stream);

/* ---------------------------------------------------------------- (add-)RMSNorm
 * add_rmsnorm_forward_kernel / add_rmsnorm_backward_kernel
 * (solution/kernels/add_rmsnorm.py:37-81) and the Qwen2 RMSNorm kernels
 * (solution/kernels/rmsnorm.py:42-102).  Rows are contiguous with row stride H
 * unless a stride argument says otherwise; weight has element stride w_stride.
 * The sum dtype S = promote(residual, delta); y is stored in y_dtype. */
int sb_add_rmsnorm_fwd(const void* residual, int r_dtype, const void* delta, int d_dtype,
                       const void* weight, int w_dtype, int64_t w_stride, void* s, void* y,
                       int y_dtype, float* rstd, int64_t rows, int64_t h, float eps,
                       void* stream);
/* gs / gy may be NULL (no upstream on that output); dr / dd may be NULL. */
int sb_add_rmsnorm_bwd(const void* s, int s_dtype, const void* weight, int w_dtype,
                       int64_t w_stride, const float* rstd, const void* gs, int gs_dtype,
                       int64_t gs_row, int64_t gs_col, const void* gy, int gy_dtype,
                       int64_t gy_row, int64_t gy_col, void* dr, int dr_dtype, void* dd,
                       int dd_dtype, int64_t rows, int64_t h, void* stream);
int sb_rmsnorm_fwd(const void* x, int x_dtype, int64_t x_row, const void* weight, int w_dtype,
                   int64_t w_stride, void* y, int y_dtype, float* rstd, int64_t rows,
                   int64_t h, float eps, void* stream);
int sb_rmsnorm_input_grad(const void* x, int x_dtype, int64_t x_row, const void* weight,
                          int w_dtype, int64_t w_stride, const void* g, int g_dtype,
                          int64_t g_row, int64_t g_col, const float* rstd, void* dx,
                          int64_t rows, int64_t h, void* stream);
/* Two-stage, atomic-free dgamma = sum_rows(g * cast_X(x * rstd)); when
 * exact_half != 0 each product is rounded to fp16 first (rmsnorm.py:73-102).
 * workspace: sb_rmsnorm_weight_grad_workspace_bytes(rows, h). */
int sb_rmsnorm_weight_grad(const void* x, int x_dtype, int64_t x_row, const void* g,
                           int g_dtype, int64_t g_row, int64_t g_col, const float* rstd,
                           void* dw, int dw_dtype, int64_t rows, int64_t h, int exact_half,
                           void* workspace, size_t workspace_bytes, void* stream);
size_t sb_rmsnorm_weight_grad_workspace_bytes(int64_t rows, int64_t h);

/* ---------------------------------------------------------------- Fused linear CE
 * _FrozenLinearCrossEntropy (solution/kernels/cross_entropy.py:133-211):
 * logits = fp16(hidden . W^T) are formed tile by tile on the tensor cores and
 * never written to memory.  Forward returns per-row loss (0 where ignored),
 * entropy, first argmax and lse (fp32 / int64).  hidden fp16 [t, h] row-major;
 * weight fp16 [v, h] row-major; targets int64 [t]; a target outside [0, v) that
 * is not ignore_index raises SB_EINVAL from sb_ce_check_targets. */
int sb_ce_forward(const uint16_t* hidden, int64_t t, int64_t h, const uint16_t* weight,
                  int64_t v, const int64_t* targets, int64_t ignore_index, float* loss,
                  float* entropy, int64_t* argmax, float* lse, void* workspace,
                  size_t workspace_bytes, void* stream);
size_t sb_ce_forward_workspace_bytes(int64_t t, int64_t h, int64_t v);
/* Vocabulary-sharded forward: sb_ce_forward over this rank's rows of the head,
 * plus row_max[t], the largest (fp16-rounded) logit of the shard, which the
 * cross-rank merge needs for the global first argmax.  Targets that belong to
 * another shard are passed as -1: they match no column, so the shard
 * contributes only its softmax terms (no counterpart in the reference, which
 * runs on one GPU; the per-shard statistics are those of cross_entropy.py:51-105). */
int sb_ce_forward_shard(const uint16_t* hidden, int64_t t, int64_t h, const uint16_t* weight,
                        int64_t v, const int64_t* targets, int64_t ignore_index, float* loss,
                        float* entropy, int64_t* argmax, float* lse, float* row_max,
                        void* workspace, size_t workspace_bytes, void* stream);
/* dhidden[t, h] (dtype dh_dtype) of sum_rows(grad[i] * loss[i]); ignored rows
 * get exact zeros and never touch their (possibly non-finite) grad. */
int sb_ce_backward(const uint16_t* hidden, int64_t t, int64_t h, const uint16_t* weight,
                   int64_t v, const int64_t* targets, int64_t ignore_index, const float* lse,
                   const float* grad, void* dhidden, int dh_dtype, void* workspace,
                   size_t workspace_bytes, void* stream);
size_t sb_ce_backward_workspace_bytes(int64_t t, int64_t h, int64_t v);
/* Host-visible validation of targets (replaces torch._assert_async,
 * solution/kernels/cross_entropy.py:238-240): *bad = number of targets that
 * are neither ignore_index nor in [0, v).  Synchronises `stream`. */
int sb_ce_check_targets(const int64_t* targets, int64_t t, int64_t v, int64_t ignore_index,
                        int64_t* bad, void* stream);

/* ---------------------------------------------------------------- Rotary embedding
 * rope_pair_forward_kernel / rope_pair_backward_kernel (solution/kernels/rope.py:24-105,
 * installed as Qwen2's apply_rotary_pos_emb by solution/rope.py:55-80): q [B, Hq, S, D]
 * and k [B, Hk, S, D] with element strides {batch, head, token, column} (any layout),
 * cos / sin [cs_batches (1 or B), S, D] with strides {batch, token, column = 1}.
 * Forward (backward = 0): q_out = q*cos + rotate_half(q)*sin, every product rounded to
 * q_out's dtype before the sum (eager PyTorch rounding; q_out_dtype = promote(q, cos)).
 * Backward: q / k are the output gradients and q_out / k_out receive the input
 * gradients (products rounded to their dtype).  Outputs are contiguous; a side with
 * zero heads is skipped (its pointers may be NULL).  Bit-exact. */
int sb_rope(const void* q, int q_dtype, const int64_t* q_strides, int64_t q_heads, void* q_out,
            int q_out_dtype, const void* k, int k_dtype, const int64_t* k_strides, int64_t k_heads,
            void* k_out, int k_out_dtype, const void* cos, const void* sin, int cs_dtype,
            const int64_t* cos_strides, const int64_t* sin_strides, int64_t cs_batches,
            int64_t batches, int64_t tokens, int64_t dim, int backward, void* stream);

/* ---------------------------------------------------------------- SwiGLU (element-wise)
 * swiglu_tile_engine (solution/kernels/swiglu_fused.py:21-78) on fp16 matrices
 * [rows, width] with row pitches ld_* (elements): act = g * sigmoid(g) * u, and
 * dgate = (da*u) * (p + g p (1 - p)), dup = da * g p with p = sigmoid(g), fp32 math. */
int sb_swiglu_fwd(const uint16_t* gate, int64_t ld_gate, const uint16_t* up, int64_t ld_up, uint16_t* act,
                  int64_t ld_act, int64_t rows, int64_t width, void* stream);
int sb_swiglu_bwd(const uint16_t* gate, int64_t ld_gate, const uint16_t* up, int64_t ld_up,
                  const uint16_t* grad, int64_t ld_grad, uint16_t* dgate, int64_t ld_dgate, uint16_t* dup,
                  int64_t ld_dup, int64_t rows, int64_t width, void* stream);

/* ---------------------------------------------------------------- Qwen2 MLP, fused
 * The frozen MLP of solution/mlp.py:500-593 (gate/up projections, SwiGLU, down
 * projection, and its backward) on NF4 weights, with the SwiGLU passes inside the
 * GEMM epilogues.  All fp16, 16-byte aligned; N = intermediate size.
 *
 * sb_nf4_mlp_gate_up_fwd: gate and up [N, K] (same shape, N % 128 == 0) in ONE launch:
 *   gate_up[m, 2N] = [X.deq(Wg)^T | X.deq(Wu)^T] (+ lora_a[m, r] . lora_b[2N, r]^T),
 *   act[m, N] = SwiGLU(gate, up) of the fp16-rounded gate/up.  For two adapters of
 *   rank r0, lora_a = [s X.Ag^T | s X.Au^T] and lora_b = [[Bg, 0]; [0, Bu]] (r = 2 r0).
 * sb_nf4_mlp_down_dx: down [K_h, N]; dact = dY[m, K_h] . deq(Wd) (+ LoRA as in
 *   sb_nf4_linear_dx) rounded to fp16, then dgate_up[m, 2N] = [dgate | dup] against
 *   gate_up[m, 2N] (N % 64 == 0).
 * sb_nf4_linear_dx2: the input gradient of two projections of one input, as one
 *   reduction: dX[m, K] = dY2[m, 2N] . [deq(W1); deq(W2)] (+ lora_a[m, r] . lora_b[K, r]^T),
 *   W1, W2 [N, K] (N % 64 == 0); workspace: sb_nf4_linear_dx2_workspace_bytes(m, N, K). */
int sb_nf4_mlp_gate_up_fwd(const uint16_t* x, int64_t m, const sb_nf4_weight* gate, const sb_nf4_weight* up,
                           const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* gate_up,
                           uint16_t* act, void* stream);
int sb_nf4_mlp_down_dx(const uint16_t* dy, int64_t m, const sb_nf4_weight* down, const uint16_t* lora_a,
                       const uint16_t* lora_b, int r, const uint16_t* gate_up, uint16_t* dgate_up, void* stream);
size_t sb_nf4_linear_dx2_workspace_bytes(int64_t m, int64_t n_out, int64_t k_in);
int sb_nf4_linear_dx2(const uint16_t* dy2, int64_t m, const sb_nf4_weight* w1, const sb_nf4_weight* w2,
                      const uint16_t* lora_a, const uint16_t* lora_b, int r, uint16_t* dx, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- Unpadding
 * Right-padded batches packed to their real tokens (solution/unpad.py: mask rules
 * :51-72, _batch_metadata :164-183, _indices_from_lengths :186-200, _pack :149-150,
 * _scatter :153-161).  mask [batch, seq] with mask_dtype 0 int64, 1 int32, 2 uint8 /
 * bool, 3 fp16, 4 fp32; labels [batch, seq] int64 or NULL.
 * sb_unpad_metadata: cu_seqlens[0..batch] = exclusive prefix of the per-row real
 *   lengths and cu_seqlens[batch + 1] = validity bits (1 a value other than 0/1,
 *   2 a one after a zero, 4 a padded label other than ignore_index, 8 an empty
 *   row); cu_seqlens holds batch + 2 int32.  workspace: sb_unpad_workspace_bytes(batch).
 * sb_unpad_pack: packed[i] = x[b, i - cu[b]] for the `rows` real rows, rows of
 *   row_bytes bytes.  sb_unpad_scatter: out[b, t] = packed[cu[b] + t] for t below
 *   the row's length, zero bytes elsewhere.  Byte copies (16-byte when aligned). */
size_t sb_unpad_workspace_bytes(int64_t batch);
int sb_unpad_metadata(const void* mask, int mask_dtype, const int64_t* labels, int64_t ignore_index, int64_t batch,
                      int64_t seq, int32_t* cu_seqlens, void* workspace, size_t workspace_bytes, void* stream);
int sb_unpad_pack(const void* x, int64_t batch, int64_t seq, int64_t row_bytes, const int32_t* cu_seqlens,
                  int64_t rows, void* packed, void* stream);
int sb_unpad_scatter(const void* packed, int64_t batch, int64_t seq, int64_t row_bytes, const int32_t* cu_seqlens,
                     void* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SOUPSUCK_B200_H */
