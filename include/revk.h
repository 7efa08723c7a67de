/* librevk — C ABI of the B200 (sm_100a) kernels behind the `reversability_b200`
 * package, a drop-in for the reversible-Transformer hot path of
 * LokeshJatangi/Reversability (`src/reversibility`).
 *
 * Conventions (all entry points):
 *  - Every pointer is a DEVICE pointer owned by the caller; the library never
 *    allocates device memory. Workspaces (RMSNorm weight-gradient partials,
 *    GEMM split partials) are passed in by the caller with their size.
 *  - Sizes and leading dimensions are element counts (int64_t).
 *  - RMSNorm, SwiGLU and the reconstruct steps accept zero rows (elements):
 *    they return RK_OK without touching the data arrays, which may then be
 *    null (an empty torch tensor has a null data pointer). The RMSNorm
 *    backward still sets dw to zero unless it accumulates.
 *  - `stream` is a cudaStream_t passed as void*; launches are stream ordered
 *    and nothing here synchronises the host.
 *  - Return value: RK_OK (0) or one of the RK_ERR_* codes below. No C++
 *    exception crosses this boundary.
 *  - Device-side bounded waits that give up set bits in a device status word;
 *    read (and clear) it with rk_device_status_read().
 * Each declaration names the reference code it replaces (path:line in the
 * reference repository).
 */
#ifndef REVK_H
#define REVK_H
#include <stdint.h>

#if defined(__GNUC__)
#define RK_API __attribute__((visibility("default")))
#else
#define RK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
enum { RK_F32 = 0, RK_BF16 = 1, RK_F16 = 2 };

/* status codes */
enum {
  RK_OK = 0,
  RK_ERR_ARG = 1,         /* null pointer, negative or inconsistent size */
  RK_ERR_ALIGN = 2,       /* pointer or leading dimension breaks a vector/TMA alignment rule */
  RK_ERR_DTYPE = 3,       /* dtype combination not supported */
  RK_ERR_LAUNCH = 4,      /* CUDA launch or driver call failed */
  RK_ERR_UNSUPPORTED = 5, /* shape outside what the kernel implements (e.g. width > 1024) */
  RK_ERR_WORKSPACE = 6,   /* caller workspace too small */
  RK_ERR_DEVICE = 7,      /* device status word non-zero (a bounded wait gave up) */
  RK_ERR_SCRATCH = 8      /* request larger than an allocation-free entry point's static scratch */
};

/* device status bits */
enum {
  RK_DEV_GEMM_TIMEOUT = 1u << 0,
  RK_DEV_ATTN_TIMEOUT = 1u << 1,
  RK_DEV_CE_LABEL = 1u << 2,    /* a cross-entropy label outside [0, vocab) and != ignore_index */
  RK_DEV_EMB_INDEX = 1u << 3    /* an embedding id outside [0, vocab) */
};

RK_API int rk_abi_version(void);
/* Number of kernel launches this library has issued in the process (host-side
 * counter; a CUDA-graph replay re-runs captured launches without counting). */
RK_API unsigned long long rk_launch_count(void);
RK_API const char* rk_status_string(int status);
/* Copies the device status word of the current device to *out and clears it.
 * Synchronises `stream`. */
RK_API int rk_device_status_read(unsigned int* out, void* stream);

/* ------------------------------------------------------------------ RMSNorm
 * Replaces kernels_v3.py:9-17 (_rms_forward) launched from kernels_v3.py:60
 * (FusedRMSNorm.forward) and nn.RMSNorm in model.py:62-64.
 * y[r,c] = (x[r,c] * rstd[r]) * w[c], rstd[r] = rsqrt(mean_c x[r,c]^2 + eps).
 * x, y: row-major [rows, width] with leading dims ldx, ldy; dtypes RK_F32/RK_BF16/RK_F16.
 * w: fp32 [width]. rstd: fp32 [rows] (may be NULL). width <= 1024. */
RK_API int rk_rmsnorm_fwd(const void* x, int x_dtype, int64_t ldx, const float* w, void* y, int y_dtype, int64_t ldy,
                   float* rstd, int64_t rows, int64_t width, float eps, void* stream);

/* Replaces kernels_v3.py:19-48 (_rms_dx, _rms_dw_partials, _rms_dw_reduce)
 * launched from kernels_v3.py:71-73 (FusedRMSNorm.backward).
 * dx = (dy*w - x * sum(dy*w*x)/width * rstd^2) * rstd ; dw = sum_rows dy * (x*rstd).
 * dx may alias nothing else. dw (fp32 [width]) is overwritten, or accumulated
 * into when accumulate_dw != 0. dw_partial: fp32 workspace of at least
 * rk_rmsnorm_bwd_workspace(rows, width) bytes. */
RK_API int64_t rk_rmsnorm_bwd_workspace(int64_t rows, int64_t width);
RK_API int rk_rmsnorm_bwd(const void* x, int x_dtype, int64_t ldx, const float* w, const float* rstd, const void* dy,
                   int dy_dtype, int64_t lddy, void* dx, int dx_dtype, int64_t lddx, float* dw, int accumulate_dw,
                   float* dw_partial, int64_t workspace_bytes, int64_t rows, int64_t width, void* stream);

/* Residual add fused into RMSNorm: s = x + a (fp32), y = rmsnorm(s) * w
 * (model.py:67-68, reversible.py:18: mlp_norm(x + attention)). x fp32, a in
 * a_dtype, y in y_dtype, rows contiguous (ld = width, width % 4 == 0).
 * sum_out (fp32, may be NULL) receives s; rstd may be NULL. */
RK_API int rk_add_rmsnorm_fwd(const float* x, const void* a, int a_dtype, const float* w, void* y, int y_dtype,
                              float* sum_out, float* rstd, int64_t rows, int64_t width, float eps, void* stream);
/* RMSNorm backward (fp32 input, rows contiguous) with the reversible step's
 * cotangent bookkeeping fused into its epilogue: dx_out = dx + residual
 * (residual may be NULL); if lp_out is not NULL it receives, in lp_dtype,
 * round(lp_add + round(dx)) when lp_add is given (the low-precision sum
 * autograd forms when a bf16 tensor has two consumers) or
 * round(round(dx_out) * lp_scale) otherwise (rk_cast_scale of the total;
 * lp_scale = 1 is the plain cast). Workspace as rk_rmsnorm_bwd. */
RK_API int rk_rmsnorm_bwd_fused(const float* x, const float* w, const float* rstd, const void* dy, int dy_dtype,
                                const float* residual, const void* lp_add, void* lp_out, int lp_dtype, float lp_scale,
                                float* dx_out, float* dw, int accumulate_dw, float* dw_partial,
                                int64_t workspace_bytes, int64_t rows, int64_t width, void* stream);
/* The weight-gradient reduction of rk_rmsnorm_bwd_fused on its own: called
 * with dw = NULL, rk_rmsnorm_bwd_fused leaves its per-CTA partials in
 * dw_partial; this sums them in the same fixed order into dw (dw += sum when
 * accumulate_dw != 0), on any stream ordered after it. rows and width are
 * those of the backward that wrote the partials. */
RK_API int rk_rmsnorm_dw_reduce(const float* dw_partial, int64_t rows, int64_t width, float* dw, int accumulate_dw,
                                void* stream);

/* Allocation-free rk_rmsnorm_bwd. It has no counterpart in the reference: it
 * exists for callers that cannot supply device workspace — foreign-function
 * hosts without a device allocator, plugins whose framework allocator owns all
 * device memory — and is otherwise the same computation with the same arguments minus dw_partial/workspace_bytes.
 * The weight-gradient partials live in a static device array of 2,424,832
 * bytes (592 x 1024 fp32), held on every GPU that loads the library until exit;
 * widths above 1024 return RK_ERR_SCRATCH. The library allocates nothing here.
 * The first call on each device looks the array's address up (with that device
 * current); make that first call before any stream capture. All calls share
 * the one array, so calls that overlap on the GPU (different streams, or
 * different host threads, on one device) race; serialise them. */
RK_API int rk_rmsnorm_bwd_noalloc(const void* x, int x_dtype, int64_t ldx, const float* w, const float* rstd,
                                  const void* dy, int dy_dtype, int64_t lddy, void* dx, int dx_dtype, int64_t lddx,
                                  float* dw, int accumulate_dw, int64_t rows, int64_t width, void* stream);

/* ------------------------------------------------------------------ SwiGLU
 * Replaces kernels.py:88-95 (_swiglu_forward) launched from kernels.py:120
 * (FusedSwiGLU.forward) and MLP.forward's silu(gate)*value (model.py:55-56).
 * u: [rows, 2*width] (gate = first width columns, value = last width columns).
 * h[r,c] = round(silu(gate)) * value, computed in fp32 and stored in `dtype`. */
RK_API int rk_swiglu_fwd(const void* u, void* h, int dtype, int64_t rows, int64_t width, void* stream);

/* Replaces kernels.py:98-110 (_swiglu_backward), launched from kernels.py:130.
 * du[:, :width]  = round(dh*value) * sig*(1 + gate*(1-sig))
 * du[:, width:]  = dh * round(silu(gate)). */
RK_API int rk_swiglu_bwd(const void* u, const void* dh, void* du, int dtype, int64_t rows, int64_t width, void* stream);

/* ------------------------------------------------------------ Reconstruct
 * Replaces inverse_pair (reversible.py:28-32) for the midpoint recurrence:
 * x_prev[i] = x_next[i] - round_F(coeff * force[i]), coeff = 2h, computed the
 * way autocast does it (scaled force rounded to the force dtype, then an fp32
 * subtraction). x_next/x_prev fp32 [n]; force dtype RK_F32/RK_BF16/RK_F16.
 * x_prev may alias x_next. */
RK_API int rk_reconstruct_midpoint(const float* x_next, const void* force, int force_dtype, float coeff, float* x_prev,
                            int64_t n, void* stream);
/* Midpoint step with the force given as its two sublayer outputs:
 * F = round(a + m) (attention + MLP, reversible.py:18, in the force dtype),
 * x_prev = x_next - round(coeff * F). coeff = 2h reconstructs (inverse_pair);
 * coeff = -2h applies the forward update p + 2h*F (forward_pair). */
RK_API int rk_reconstruct_midpoint_sum(const float* x_next, const void* a, const void* m, int dtype, float coeff,
                                       float* x_prev, int64_t n, void* stream);
/* out = round(round(x) * scale) in out_dtype: an fp32 cotangent cast to the
 * compute dtype and scaled there (the backward of `2 * h * F` under autocast,
 * reversible.py:22). */
RK_API int rk_cast_scale(const float* x, void* out, int out_dtype, float scale, int64_t n, void* stream);
/* Hamiltonian-Euler inverse half-step (reversible.py:30-32):
 * state_prev[i] = state[i] - sublayer_out[i] (p_prev = p - M(q); q_prev = q - A(p_prev)). */
RK_API int rk_reconstruct_euler(const float* state, const void* sublayer_out, int out_dtype, float* state_prev, int64_t n,
                         void* stream);

/* ------------------------------------------------------------------ GEMMs
 * Replace F.linear (cuBLAS) inside CausalSelfAttention.qkv/.proj and
 * MLP.up/.down (model.py:37,45,55-56) and its autograd backward.
 * Operand dtype `dtype` is RK_BF16 or RK_F16 (tcgen05 tensor cores, fp32
 * accumulation in tensor memory) or RK_F32 (CUDA-core fp32 path used by the
 * fp32 parity configuration). Row-major everywhere; ld* are row strides.
 *
 * fprop: Y[M,N] = X[M,K] . W[N,K]^T            (nn.Linear forward)
 * dgrad: DX[M,K] = DY[M,N] . W[N,K]            (grad wrt the Linear input)
 * wgrad: DW[N,K] (+)= DY[M,N]^T . X[M,K]       (grad wrt the weight, fp32 out)
 * out_dtype: dtype of Y/DX (RK_F32, RK_BF16 or RK_F16).
 * For bf16/f16 operands the row strides in bytes must be multiples of 16 and
 * the base pointers 16-byte aligned (TMA rule).
 * wgrad splits the M reduction into fixed slices written to `workspace`
 * (fp32) and summed in a fixed order, so results are deterministic; size it
 * with rk_gemm_wgrad_workspace(). accumulate != 0 adds into DW. */
RK_API int rk_gemm_fprop(const void* x, int64_t ldx, const void* w, int64_t ldw, void* y, int64_t ldy, int64_t M,
                  int64_t N, int64_t K, int dtype, int out_dtype, void* stream);
RK_API int rk_gemm_dgrad(const void* dy, int64_t lddy, const void* w, int64_t ldw, void* dx, int64_t lddx, int64_t M,
                  int64_t N, int64_t K, int dtype, int out_dtype, void* stream);
/* Attention output projection's dgrad with the attention backward's
 * D = rowsum(dO * O) in its epilogue (model.py:45 backward and the D term of
 * F.scaled_dot_product_attention's backward): DX[M,K] = DY[M,N] . W[N,K] as
 * rk_gemm_dgrad (16-bit, dtype), and dsum[b, h, t] = sum over head h's
 * columns of DX[b*T + t] * O[b*T + t] with O [M, K], K = H * 32 or H * 64,
 * M = B * T;
 * bit-identical to rk_gemm_dgrad followed by rk_attn_bwd_piece(0). Returns
 * RK_ERR_UNSUPPORTED when the layout does not fit the TMA epilogue. */
/* Sublayer output projection with the reversible state update in its
 * epilogue (replaces the projection + inverse_pair / forward_pair arithmetic of
 * reversible.py:21-32 and optimized.py:31-32):
 *   out[M,N] = state[M,N] - round(coeff * round(round(x[M,K] . W[N,K]^T) + addend[M,N]))
 * with addend null meaning no addend; rounding to the 16-bit dtype (bf16/f16)
 * where autocast rounds, the subtraction in fp32. Midpoint: the MLP down
 * projection with addend = the attention output a, coeff = 2h (reconstruction)
 * or -2h (forward). Euler: coeff = 1 or -1 without an addend. The sublayer
 * output never reaches global memory; out may equal state. Bit-identical to
 * rk_gemm_fprop followed by rk_reconstruct_midpoint_sum / rk_reconstruct_midpoint.
 * N % 32 == 0 (else RK_ERR_UNSUPPORTED); state/out 16-byte aligned with row
 * strides that are multiples of 4 elements, addend with strides multiple of 8. */
RK_API int rk_gemm_fprop_reconstruct(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* state,
                              int64_t lds, const void* addend, int64_t lda, float coeff, float* out, int64_t ldo,
                              int64_t M, int64_t N, int64_t K, int dtype, void* stream);
/* rk_gemm_fprop_reconstruct followed, in the same pass, by the RMSNorm forward
 * of the updated state (the next sublayer's input norm, model.py:62-64;
 * replaces rk_rmsnorm_fwd on an fp32 state, or rk_add_rmsnorm_fwd when the
 * state update is the residual add x + a: coeff = -1, no addend):
 *   y[M,N] = round((out * rstd) * norm_w), rstd[M] = rsqrt(mean(out^2) + eps)
 * bit-identical to the standalone norm on `out`. rstd may be NULL. If low is
 * not NULL it also receives round(x . W^T) (what rk_gemm_fprop stores; the
 * residual branch's a). N must be 256 (RK_ERR_UNSUPPORTED otherwise); y, low
 * and norm_w 16-byte aligned, ldy and ldl multiples of 8. */
RK_API int rk_gemm_fprop_reconstruct_norm(const void* x, int64_t ldx, const void* w, int64_t ldw, const float* state,
                                          int64_t lds, const void* addend, int64_t lda, float coeff, float* out,
                                          int64_t ldo, void* low, int64_t ldl, const float* norm_w, float eps, void* y,
                                          int64_t ldy, float* rstd, int64_t M, int64_t N, int64_t K, int dtype,
                                          void* stream);
RK_API int rk_gemm_dgrad_dsum(const void* dy, int64_t lddy, const void* w, int64_t ldw, void* dx, int64_t lddx,
                              int64_t M, int64_t N, int64_t K, int dtype, const void* o, int64_t ldo, float* dsum,
                              int64_t T, int64_t H, void* stream);
/* MLP up projection with SwiGLU fused into the epilogue (model.py:55-56):
 * u = X[M,K] . W_up[2ff,K]^T, h[M,ff] = round(silu(u[:, :ff])) * u[:, ff:] with
 * the same rounding as rk_swiglu_fwd on a bf16/f16 u. If u is not NULL it also
 * receives u itself (the backward needs it). bf16/f16 only; ff % 128 == 0. */
RK_API int rk_gemm_fprop_swiglu(const void* x, int64_t ldx, const void* w_up, int64_t ldw, void* h, int64_t ldh,
                                void* u, int64_t ldu, int64_t M, int64_t ff, int64_t K, int dtype, void* stream);
/* MLP down projection's dgrad with the SwiGLU backward fused into the
 * epilogue (model.py:55-56 backward): dh = round(DY[M,N] . W_down[N,ff]) and
 * du[M,2ff] = rk_swiglu_bwd(u, dh), bit-identical to rk_gemm_dgrad followed by
 * rk_swiglu_bwd; dh is never written. u/du hold the gate half in columns
 * [0, ff) and the value half in [ff, 2ff). bf16/f16 only; ff % 64 == 0. */
RK_API int rk_gemm_dgrad_swiglu(const void* dy, int64_t lddy, const void* w, int64_t ldw, const void* u, int64_t ldu,
                                void* du, int64_t lddu, int64_t M, int64_t ff, int64_t N, int dtype, void* stream);
RK_API int64_t rk_gemm_wgrad_workspace(int64_t M, int64_t N, int64_t K);
RK_API int rk_gemm_wgrad(const void* dy, int64_t lddy, const void* x, int64_t ldx, float* dw, int64_t lddw, int64_t M,
                  int64_t N, int64_t K, int dtype, int accumulate, float* workspace, int64_t workspace_bytes,
                  void* stream);

/* ------------------------------------------------------------- Attention
 * Replaces F.scaled_dot_product_attention(q, k, v, is_causal=True) and the
 * q/k/v view/transpose plumbing of CausalSelfAttention.forward (model.py:35-45).
 * qkv: [B*T, ldq] rows holding q | k | v (each H*HD wide, head h at h*HD), i.e.
 * the qkv Linear output as is. out: [B*T, ldo], head h at columns h*HD (the
 * proj Linear input). lse: fp32 [B, H, T] row log-sum-exp saved for backward
 * (base 2 of the scaled scores for bf16/f16, natural log for fp32).
 * dtype RK_BF16/RK_F16 (tensor cores, HD 32 or 64) or RK_F32 (CUDA cores).
 * Softmax scale 1/sqrt(HD). Deterministic (no atomics). */
RK_API int rk_attn_fwd(const void* qkv, int64_t ldq, void* out, int64_t ldo, float* lse, int64_t B, int64_t H,
                       int64_t HD, int64_t T, int dtype, void* stream);
/* Backward: dqkv [B*T, lddq] receives dq | dk | dv in the qkv layout.
 * dout has the layout of out (same ldo). dsum: fp32 [B, H, T] scratch
 * (rowsum(dout*out)). */
RK_API int rk_attn_bwd(const void* qkv, int64_t ldq, const void* out, const void* dout, int64_t ldo,
                       const float* lse, float* dsum, void* dqkv, int64_t lddq, int64_t B, int64_t H, int64_t HD,
                       int64_t T, int dtype, void* stream);
/* The backward in pieces (bf16/f16): piece 0 writes dsum = rowsum(dout*out),
 * piece 1 dq and piece 2 dk|dv (both read dsum). Pieces 1 and 2 touch disjoint
 * columns of dqkv and may run concurrently on two streams after piece 0. */
RK_API int rk_attn_bwd_piece(int piece, const void* qkv, int64_t ldq, const void* out, const void* dout,
                             int64_t ldo, const float* lse, float* dsum, void* dqkv, int64_t lddq, int64_t B,
                             int64_t H, int64_t HD, int64_t T, int dtype, void* stream);

/* ---------------------------------------------------------- Cross-entropy
 * Replaces F.cross_entropy(logits, labels, ignore_index=-100, reduction="sum")
 * and its backward (train_baseline.py:262; Triton variant kernels.py:14-85).
 * logits: [rows, ld] (vocab valid columns), dtype RK_F32/RK_BF16/RK_F16.
 * loss_rows[r] = logsumexp(logits[r]) - logits[r, labels[r]] (0 for ignored rows).
 * dlogits[r, c] = (softmax(logits[r])[c] - [c == labels[r]]) * scale, zero rows
 * for ignored labels, where scale = grad_scale * (*grad_scale_dev) when
 * grad_scale_dev (a device fp32 scalar, e.g. 1/update_targets kept on the GPU
 * so a captured CUDA graph can be replayed with a new denominator) is not
 * NULL, else grad_scale. dlogits may alias logits (in place). fp32 math. */
RK_API int rk_cross_entropy_fwd_bwd(const void* logits, int64_t ld, int64_t vocab, const int64_t* labels,
                                    int64_t rows, float grad_scale, const float* grad_scale_dev, float* loss_rows,
                                    void* dlogits, int64_t ldd, int dtype, int ignore_index, void* stream);

/* ------------------------------------------------ Softmax head (fused CE)
 * The vocabulary head and its cross-entropy with no pass of their own over the
 * logits; together they replace the head Linear, F.cross_entropy(...,
 * reduction="sum") and their backward (model.py:104, train_baseline.py:262,
 * optimized_v3.py cached_head_backward). Blocks b are 128 columns wide.
 *   rk_head_fprop : expo[M, V] = exp(x - m_b) (bf16/f16) where x = hidden . W^T
 *                   rounded to the compute type and m_b the max of x over the
 *                   row's block b; stats[M][width] float2 = (m_b, sum of exp)
 *                   with width = rk_head_stats_width(V); xlabel[r] = x at the
 *                   row's label (rows whose label is in [0, V));
 *   rk_head_loss  : loss_rows[r] = lse - x[label] (0 for ignore_index),
 *                   rowc[r] float4 = (-lse*log2(e), s, (exp(x[label]-lse)-1)*s, 0)
 *                   with s = grad_scale * (*grad_scale_dev), and the per-block
 *                   factors fcoef[b * fcoef_ld + r] = exp(m_b - lse) * s
 *                   ([width][fcoef_ld >= rows] floats); all 0 for ignored rows;
 *                   a label outside [0, V) sets RK_DEV_CE_LABEL and the row is
 *                   ignored;
 *   rk_head_dgrad : dhidden[M, K] = dlogits . W, and
 *   rk_head_wgrad : dW[V, K] (+)= dlogits^T . hidden, where
 *                   dlogits = (softmax(x) - onehot(label)) * s is formed inside
 *                   the GEMM as expo * fcoef, the label entry taken from rowc
 *                   (never written to global memory). */
RK_API int64_t rk_head_stats_width(int64_t vocab);
RK_API int rk_head_fprop(const void* hidden, int64_t ldh, const void* w, int64_t ldw, const int64_t* labels,
                         void* expo, int64_t lde, float* stats, float* xlabel, int64_t M, int64_t V, int64_t K,
                         int dtype, void* stream);
RK_API int rk_head_loss(const float* stats, int64_t width, const float* xlabel, const int64_t* labels, int64_t rows,
                        int64_t V, float grad_scale, const float* grad_scale_dev, float* loss_rows, float* rowc,
                        float* fcoef, int64_t fcoef_ld, int ignore_index, void* stream);
RK_API int rk_head_dgrad(const void* expo, int64_t lde, const float* fcoef, int64_t fcoef_ld, const float* rowc,
                         const int64_t* labels, const void* w, int64_t ldw, void* dx, int64_t lddx, int64_t M,
                         int64_t V, int64_t K, int dtype, int out_dtype, void* stream);
/* rk_head_dgrad with the vocabulary reduction split into slices when the
 * output has fewer 128 x 256 tiles than the GPU has SMs (cfg2: 116 tiles),
 * so every SM works: fp32 partial slices in `workspace` (at least
 * rk_head_dgrad_workspace(M, V, K) bytes, 16-byte aligned; 0 = no split for
 * this shape), then a fixed-order sum into dx (deterministic; the sum order
 * differs from the unsplit kernel's, so results agree to fp32 rounding of
 * the partials). Falls back to rk_head_dgrad when the workspace is short, the
 * shape needs no split, or K / lddx are not multiples of 4. */
RK_API int64_t rk_head_dgrad_workspace(int64_t M, int64_t V, int64_t K);
RK_API int rk_head_dgrad_ws(const void* expo, int64_t lde, const float* fcoef, int64_t fcoef_ld, const float* rowc,
                            const int64_t* labels, const void* w, int64_t ldw, void* dx, int64_t lddx, int64_t M,
                            int64_t V, int64_t K, int dtype, int out_dtype, float* workspace,
                            int64_t workspace_bytes, void* stream);
RK_API int rk_head_wgrad(const void* expo, int64_t lde, const float* fcoef, int64_t fcoef_ld, const float* rowc,
                         const int64_t* labels, const void* x, int64_t ldx, float* dw, int64_t lddw, int64_t M,
                         int64_t V, int64_t K, int dtype, int accumulate, void* stream);

/* -------------------------------------------------------- Clip + AdamW
 * Replace torch.nn.utils.clip_grad_norm_(params, max_norm) and
 * torch.optim.AdamW(lr, betas, weight_decay).step() over the parameters of the
 * whole model held in one flat fp32 buffer (train_baseline.py:152-154,272,280).
 * scalars: device fp32[8]: [0] lr (set by the caller), [1] step count
 * (incremented by prepare), [2] gradient norm, [3] clip coefficient,
 * [4..6] derived per-step constants. prepare computes the global norm
 * deterministically (fixed-order two-pass reduction) into scalars; step applies
 * the clip coefficient and the AdamW update in one pass and, if params_c is
 * non-NULL, writes the updated parameters in c_dtype (RK_BF16/RK_F16) too. */
RK_API int64_t rk_clip_adamw_workspace(void);
RK_API int rk_clip_adamw_prepare(const float* grads, int64_t n, float max_norm, float beta1, float beta2,
                                 float weight_decay, float* workspace, int64_t workspace_bytes, float* scalars,
                                 void* stream);
RK_API int rk_adamw_step(float* params, const float* grads, float* exp_avg, float* exp_avg_sq, void* params_c,
                         int c_dtype, int64_t n, const float* scalars, float beta1, float beta2, float eps,
                         void* stream);

/* ------------------------------------------------------------- Embedding
 * Replace the token + learned position embedding of BaselineLM.forward /
 * ReversibleLM.forward (model.py:98-101, reversible.py:105-106) and its
 * backward. ids: int64 [rows] (rows = B*T, row r at position r % T);
 * tok fp32 [V, d]; pos fp32 [>= T, d]; out fp32 [rows, d].
 * Backward accumulates dx (+ dx2 if not NULL; the two cotangents the boundary
 * p = q = embedding receives, reversible.py:91) into g_tok [V, d] and g_pos [>= T, d] (fp32) in a fixed
 * order: rows are grouped by id with a stable radix sort and each group is
 * summed in row order, so results are bitwise reproducible. workspace: at
 * least rk_embedding_bwd_workspace(rows, V) bytes, 16-byte aligned. d must be
 * a multiple of 4. */
RK_API int rk_embedding_fwd(const int64_t* ids, const float* tok, const float* pos, float* out, int64_t rows,
                            int64_t T, int64_t d, int64_t V, void* stream);
RK_API int64_t rk_embedding_bwd_workspace(int64_t rows, int64_t V);
RK_API int rk_embedding_bwd(const int64_t* ids, const float* dx, const float* dx2, float* g_tok, float* g_pos,
                            int64_t rows, int64_t T, int64_t d, int64_t V, void* workspace, int64_t workspace_bytes,
                            void* stream);
/* rk_embedding_bwd in two calls. The grouping of rows by id depends on the ids
 * alone, so a caller can issue it early on another stream, off the path of
 * the backward: rk_embedding_bwd_sort writes it into `sorted` (at least
 * rk_embedding_bwd_sort_bytes(rows, V) bytes, 16-byte aligned, left untouched
 * until the matching rk_embedding_bwd_sorted has run), and
 * rk_embedding_bwd_sorted accumulates dx (+ dx2) into g_tok and g_pos from it,
 * with a workspace of at least rk_embedding_bwd_sorted_workspace(rows, d)
 * bytes. Same results as rk_embedding_bwd, bit for bit. */
RK_API int64_t rk_embedding_bwd_sort_bytes(int64_t rows, int64_t V);
RK_API int rk_embedding_bwd_sort(const int64_t* ids, int64_t rows, int64_t V, void* sorted, int64_t sorted_bytes,
                                 void* stream);
RK_API int64_t rk_embedding_bwd_sorted_workspace(int64_t rows, int64_t d);
RK_API int rk_embedding_bwd_sorted(const void* sorted, int64_t sorted_bytes, const float* dx, const float* dx2,
                                   float* g_tok, float* g_pos, int64_t rows, int64_t T, int64_t d, int64_t V,
                                   void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------------------- Reversible layer
 * One reversible Block step as a single call: the per-layer sequence of the
 * calls above (RMSNorm, QKV/proj/up/down GEMMs with their fused epilogues,
 * causal attention, their VJPs and weight gradients), issued in order on
 * `stream` (no host synchronisation, no allocation). Replaces, per layer:
 *   rk_layer_fwd_midpoint  forward_pair midpoint (reversible.py:21-23)
 *   rk_layer_fwd_euler     forward_pair Euler (reversible.py:24-25)
 *   rk_layer_bwd_midpoint  one iteration of _InverseStack.backward /
 *                          ReusedMidpoint.backward (reversible.py:47-69,
 *                          optimized.py:21-41): inverse_pair + recompute + VJP
 *   rk_layer_bwd_euler     the same for the Euler recurrence
 * with the force F(x) = A(x) + M(x + A(x)) of reversible.py:16-18 (Block of
 * model.py:59-69, bias-free). Compute dtype RK_BF16 or RK_F16 (the autocast
 * rounding points of the reference); states, cotangents, RMSNorm weights and
 * weight gradients are fp32, GEMM weights are in the compute dtype. States are
 * [tokens, d_model] row-major with tokens = batch * length (row b*length + t).
 * Weight gradients accumulate (+=) into `grads`. workspace: at least
 * rk_layer_workspace(desc, method, backward) bytes, 256-byte aligned; the
 * caller may reuse it for the next layer once the call's work is ordered
 * before (same stream). Returns RK_ERR_DTYPE for fp32 compute, which the
 * separate entry points cover. */
typedef struct rk_layer_desc {
  int64_t batch, length;      /* B, T */
  int64_t d_model, n_heads, d_ff;
  int64_t mlp_tokens;         /* MLP token tile (TiledMLP); 0 = the whole batch at once */
  int dtype;                  /* compute dtype: RK_BF16 / RK_F16 */
  float eps_attn, eps_mlp;    /* RMSNorm eps of attn_norm / mlp_norm */
  const float* attn_norm;     /* fp32 [d] */
  const void* qkv;            /* [3d, d] compute dtype (attn.qkv.weight) */
  const void* proj;           /* [d, d] (attn.proj.weight) */
  const float* mlp_norm;      /* fp32 [d] */
  const void* up;             /* [2ff, d] (mlp.up.weight: gate rows, then value rows) */
  const void* down;           /* [d, ff] (mlp.down.weight) */
} rk_layer_desc;

typedef struct rk_layer_grads {  /* fp32, Block.parameters() order */
  float *attn_norm, *qkv, *proj, *mlp_norm, *up, *down;
} rk_layer_grads;

enum { RK_METHOD_MIDPOINT = 0, RK_METHOD_EULER = 1 };

RK_API int64_t rk_layer_workspace(const rk_layer_desc* desc, int method, int backward);
/* (p, q) -> (q, q_next = p + round(2h F(q))): the next p is q itself. */
RK_API int rk_layer_fwd_midpoint(const rk_layer_desc* desc, const float* p, const float* q, float h, float* q_next,
                                 void* workspace, int64_t workspace_bytes, void* stream);
/* q_next = q + A(p), p_next = p + M(q_next). */
RK_API int rk_layer_fwd_euler(const rk_layer_desc* desc, const float* p, const float* q, float* p_next,
                              float* q_next, void* workspace, int64_t workspace_bytes, void* stream);
/* From the states after the layer (p, q) and their cotangents (dp, dq; dp may
 * be NULL for a zero cotangent): p_prev = q - round(2h F(p)) (the previous q
 * is p itself), dq_prev = dp + J_F(p)^T round(2h round(dq)) (the previous dp
 * is dq itself). gf_in (compute dtype, may be NULL) is round(2h round(dq))
 * when the caller has it; gf_out (may be NULL) receives round(2h round(dq_prev))
 * for the layer below. */
RK_API int rk_layer_bwd_midpoint(const rk_layer_desc* desc, const rk_layer_grads* grads, const float* p,
                                 const float* q, const float* dp, const float* dq, const void* gf_in, float h,
                                 float* p_prev, float* dq_prev, void* gf_out, void* workspace,
                                 int64_t workspace_bytes, void* stream);
/* p_prev = p - M(q), q_prev = q - A(p_prev); dq_prev = dq + J_M(q)^T round(dp),
 * dp_prev = dp + J_A(p_prev)^T round(dq_prev) (dq may be NULL for zero).
 * gm_in (may be NULL) is round(dp); gm_out (may be NULL) receives
 * round(dp_prev) for the layer below. */
RK_API int rk_layer_bwd_euler(const rk_layer_desc* desc, const rk_layer_grads* grads, const float* p, const float* q,
                              const float* dp, const float* dq, const void* gm_in, float* p_prev, float* q_prev,
                              float* dp_prev, float* dq_prev, void* gm_out, void* workspace, int64_t workspace_bytes,
                              void* stream);

#ifdef __cplusplus
}
#endif
#endif /* REVK_H */
