/*
 * mea.h -- C ABI of libmea.so, the sm_100a (B200) implementation of the gated
 * causal attention block of xTimeCrystal/memory_efficient_attn_layer.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no framework types.
 * All tensors live in device memory, are contiguous and row-major, and are bf16
 * unless a parameter says fp32.  No function allocates device memory: callers
 * pass a workspace sized by the matching *_workspace_size() query.  Every
 * function returns MEA_OK (0) or an MEA_ERR_* code; mea_last_error_string()
 * describes the last failure of the calling thread.  Arguments are checked
 * before any device work is queued: a rejected call leaves the stream as it was.
 *
 * Alignment: tensors 16-byte aligned (workspaces 256-byte), except the bf16
 * weight-gradient outputs of the block backward and the bf16 dq of
 * mea_attention_backward_noalloc, which need 8 bytes; MEA_ERR_ALIGNMENT
 * otherwise.
 *
 * Device-side waits are bounded: a kernel that gives up writes a non-zero code
 * into the optional `status` word (device int, zero it before the call) and
 * returns early; read it with mea_read_status().
 *
 * Shapes (B batch, T sequence, C model dim, H heads, N head dim):
 *   T % 128 == 0, N in {32, 64, 128}, C % 128 == 0, (H*N) % 128 == 0.
 * The rotary tables factor1/factor2 are [T_max >= T, N].
 *
 * Reference interfaces cited below are files of the reference project.
 */
#ifndef MEA_H_
#define MEA_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MEA_OK = 0,
  MEA_ERR_INVALID_ARGUMENT = 1,
  MEA_ERR_UNSUPPORTED_SHAPE = 2,
  MEA_ERR_ALIGNMENT = 3,
  MEA_ERR_CUDA = 4,
  MEA_ERR_DEVICE_TIMEOUT = 5,
  MEA_ERR_UNSUPPORTED_DEVICE = 6,
  MEA_ERR_WORKSPACE = 7
};

typedef struct mea_block_dims {
  int B, T, C, H, N;
  int T_max; /* rows of the rotary tables */
  float eps; /* RMSNorm epsilon (reference default 1e-6, fast_triton_attn.py:681) */
} mea_block_dims;

/* Library version (major*10000 + minor*100 + patch). */
int mea_version(void);
/* Message of the last failure on the calling thread ("" if none). */
const char* mea_last_error_string(void);
/* MEA_OK when the current device is an sm_100 part the kernels were built for. */
int mea_device_check(void);
/* Synchronises `stream` and copies the device status word to *out; returns
 * MEA_ERR_DEVICE_TIMEOUT (with the kernel and wait site in the message) when
 * the word is non-zero. */
int mea_read_status(const int* status_dev, int* out, void* stream);
/* Self-test of the device-side failure detection; no counterpart in the
 * reference, which has none.  Launches one warp that waits on an mbarrier
 * through the same bounded wait every kernel of the library uses, with a limit
 * of limit_ns (at most 1e9).  With arrive != 0 the barrier completes at once
 * and *status is left alone; with arrive == 0 nobody arrives, the wait gives
 * up after limit_ns and records a timeout (kernel id 9, site 1) in *status,
 * exactly as a stalled kernel would.  Nothing else is in flight in that
 * kernel, so it always ends and leaves the context usable. */
int mea_selftest_wait(int* status, unsigned long long limit_ns, int arrive, void* stream);

/* ---------------------------------------------------------------- block level */

/* Bytes of workspace for mea_block_forward. */
size_t mea_forward_workspace_size(const mea_block_dims* d);
/* FusedAttentionFunction.forward (fast_triton_attn.py:374-479):
 * y[B,T,C] = o_proj(attn(norm-rope(proj(norm(x)))) * sigmoid(g)).
 * Writes lse2[B,H,T] (fp32 row log-sum-exp in log2 units), the only
 * activation kept for the backward besides x. */
int mea_block_forward(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                      const void* wg, const void* wo, const void* factor1, const void* factor2, void* y, float* lse2,
                      void* workspace, size_t workspace_bytes, int* status, void* stream);

/* Bytes of workspace for mea_block_backward. */
size_t mea_backward_workspace_size(const mea_block_dims* d);
/* FusedAttentionFunction.backward (fast_triton_attn.py:481-675): recomputes
 * the block from x and lse2, then writes dx and the five weight gradients
 * (bf16, same shapes as the weights).  dfactor1/dfactor2 (fp32 [T_max, N],
 * rows >= T zero) are written when non-NULL.  dweights_f32, when non-NULL,
 * receives the fp32 weight gradients too: [4*H*N, C] for q,k,v,g followed by
 * [C, H*N] for o. */
int mea_block_backward(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                       const void* wg, const void* wo, const void* factor1, const void* factor2, const float* lse2,
                       const void* dy, void* dx, void* dwq, void* dwk, void* dwv, void* dwg, void* dwo,
                       float* dfactor1, float* dfactor2, float* dweights_f32, void* workspace,
                       size_t workspace_bytes, int* status, void* stream);

/* mea_block_backward for data-parallel training: no counterpart in the
 * reference, whose weight gradients are exchanged after the backward.  Same
 * arguments, plus two CUDA events (cudaEvent_t, may be NULL) recorded on
 * `stream` as soon as the fp32 gradients in dweights_f32 are final: ev_dwo_ready
 * after the o_proj gradient [C, H*N] (early in the backward, before the
 * attention backward), ev_dw_ready after the q/k/v/g gradients [4*H*N, C]
 * (before the input-gradient GEMM).  A caller can start its all-reduce of each
 * part on another stream at those events, overlapping the rest of the
 * backward.  dwq .. dwo may be NULL (no bf16 copy written); dweights_f32 must
 * then be non-NULL. */
int mea_block_backward_ex(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                          const void* wg, const void* wo, const void* factor1, const void* factor2,
                          const float* lse2, const void* dy, void* dx, void* dwq, void* dwk, void* dwv, void* dwg,
                          void* dwo, float* dfactor1, float* dfactor2, float* dweights_f32, void* workspace,
                          size_t workspace_bytes, int* status, void* stream, void* ev_dwo_ready,
                          void* ev_dw_ready);

/* Keep-O variant (an ablation of the memory-saving default; it mirrors the
 * reference, which keeps the attention output, fast_triton_attn.py:463-466):
 * mea_block_forward that also writes the attention output
 * o[B,H,T,N] (bf16, before the gate) for the backward. */
int mea_block_forward_save_o(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                             const void* wg, const void* wo, const void* factor1, const void* factor2, void* y,
                             float* lse2, void* o, void* workspace, size_t workspace_bytes, int* status,
                             void* stream);
/* mea_block_backward_ex given that o (from mea_block_forward_save_o): the
 * attention recompute is skipped and the gated tile is formed from o
 * (gate_repack_kernel_bwd_recompute, fast_triton_attn.py:334-367).  Same
 * workspace size as mea_block_backward. */
int mea_block_backward_from_o(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                              const void* wg, const void* wo, const void* factor1, const void* factor2,
                              const float* lse2, const void* o, const void* dy, void* dx, void* dwq, void* dwk,
                              void* dwv, void* dwg, void* dwo, float* dfactor1, float* dfactor2,
                              float* dweights_f32, void* workspace, size_t workspace_bytes, int* status,
                              void* stream, void* ev_dwo_ready, void* ev_dw_ready);

/* ---------------------------------------------------------------- kernel level */

/* rms_norm_kernel / rms_norm_kernel_recompute (fast_triton_attn.py:12-34, :181-210):
 * xn = bf16(x * r), r[row] = rsqrt(mean(x^2) + eps).  xn may be NULL. */
int mea_rmsnorm_forward(int rows, int C, float eps, const void* x, void* xn, float* r, void* stream);

/* fused_qkvg_norm_rope_kernel(_recompute) (fast_triton_attn.py:36-144, :212-332):
 * from normalised input xn[B*T, C] write q, k (per-head RMSNorm + rotary), v and
 * sigmoid(g), each [B,H,T,N]; rq/rk[B,H,T] (fp32 inverse RMS) when non-NULL. */
int mea_qkvg_forward(const mea_block_dims* d, const void* xn, const void* wq, const void* wk, const void* wv,
                     const void* wg, const void* factor1, const void* factor2, void* q, void* k, void* v, void* gs,
                     float* rq, float* rk, int* status, void* stream);

/* ATen flash-attention forward + gate_repack_kernel (fast_triton_attn.py:425-457):
 * causal softmax(q k^T / sqrt(N)) v, times gs, repacked to gated[B,T,H*N];
 * lse2[B,H,T] fp32 (log2 units); o[B,H,T,N] (ungated output) when non-NULL. */
int mea_attention_forward(int B, int H, int T, int N, const void* q, const void* k, const void* v, const void* gs,
                          void* gated, float* lse2, void* o, int* status, void* stream);

/* F.linear / Tensor.matmul (fast_triton_attn.py:460, :578-579, :649-660):
 * out[M,N] (fp32) = sum_k A[m,k] B[n,k].  A is stored [M,K] (a_mn = 0) or
 * [K,M] (a_mn = 1) with row pitch lda; B is stored [N,K] (b_mn = 0) or [K,N]
 * (b_mn = 1) with row pitch ldb.  accumulate != 0 adds into out (split-K). */
int mea_gemm(int M, int N, int K, const void* a, long long lda, int a_mn, const void* b, long long ldb, int b_mn,
             float* out, long long ldo, int accumulate, int* status, void* stream);

/* e4m3 GEMM (no counterpart in the reference, which computes its projections
 * in bf16): out[M,N] = sum_k A[m,k] B[n,k] with A [M,K] and B [N,K] both
 * K-major e4m3 (one byte per element, row pitches lda/ldb in elements, multiples
 * of 16), fp32 accumulate, written as fp32 (out_bf16 = 0) or bf16.  No
 * scaling is applied: callers multiply by their per-tensor scales.  M % 128,
 * N % 128 and K % 128 must be zero.  The block does not use it: e4m3's 3-bit
 * mantissa costs ~3.5% max-relative error per projection GEMM, above the
 * block's 2e-2 output tolerance. */
int mea_gemm_e4m3(int M, int N, int K, const void* a, long long lda, const void* b, long long ldb, void* out,
                  long long ldo, int out_bf16, int* status, void* stream);

/* o_proj backward + gate backward (fast_triton_attn.py:576-584, :601):
 * dGated = dy * wo, then dO = dGated*gs ([B,H,T,N]), dg_pre = dGated*o*gs*(1-gs)
 * into dg[(b*T+t)*ld_dg + h*N + n], delta[B,H,T] = rowsum(dO*o) (fp32). */
int mea_gate_backward(const mea_block_dims* d, const void* dy, const void* wo, const void* o, const void* gs,
                      void* dO, void* dg, long long ld_dg, float* delta, int* status, void* stream);

/* ATen flash-attention backward (fast_triton_attn.py:586-596): adds dq into
 * dq_acc[B,H,T,N] (fp32, caller zeroes it), writes dk[B,H,T,N] and
 * dv[(b*T+t)*ld_dv + h*N + n]. */
int mea_attention_backward(int B, int H, int T, int N, const void* q, const void* k, const void* v, const void* dO,
                           const float* lse2, const float* delta, float* dq_acc, void* dk, void* dv, long long ld_dv,
                           int* status, void* stream);

/* Per-head RMSNorm + rotary backward and rotary-table gradients
 * (fast_triton_attn.py:603-639): d acc_q, d acc_k into dacc[(b*T+t)*ld_dacc +
 * {0, H*N} + h*N + n]; dfactor1/2 (fp32 [T_max, N], caller zeroes) when non-NULL. */
int mea_qk_norm_rope_backward(const mea_block_dims* d, const float* dq_acc, const void* dk, const void* q,
                              const void* k, const float* rq, const float* rk, const void* factor1,
                              const void* factor2, void* dacc, long long ld_dacc, float* dfactor1, float* dfactor2,
                              void* stream);

/* rms_norm_backward_new (fast_triton_attn.py:663-669): dx from d(xn), x and r. */
int mea_rmsnorm_backward(int rows, int C, const void* dxn, const void* x, const float* r, void* dx, void* stream);

/* ---------------------------------------------------------------- no allocation
 * No counterpart in the reference.  mea_attention_backward for callers that
 * cannot allocate device memory (for example a plugin whose execute callback
 * may not call cudaMalloc, or code handed only its input and output buffers):
 * the fp32 dQ accumulator lives in a 16 MiB array inside the library (held by
 * every GPU that loads it), so B*H*T*N must not exceed 4,194,304; larger
 * problems return MEA_ERR_UNSUPPORTED_SHAPE.  dq is written as bf16
 * [B,H,T,N] (8-byte aligned); dk, dv as in mea_attention_backward.  All calls share that array:
 * calls that overlap on the GPU race.  The first call on a device looks up the
 * array's address; make it before any stream capture. */
int mea_attention_backward_noalloc(int B, int H, int T, int N, const void* q, const void* k, const void* v,
                                   const void* dO, const float* lse2, const float* delta, void* dq, void* dk,
                                   void* dv, long long ld_dv, int* status, void* stream);

/* ---------------------------------------------------------------- optimizer
 * No counterpart in the reference, whose module (README.md:6-68) leaves the
 * weight update to the caller's optimizer.  One AdamW step, in the order
 * torch.optim.AdamW applies it (decoupled weight decay, bias-corrected
 * moments, step counted from 1), over n contiguous fp32 master weights and
 * their two moments, all updated in place, with g = grad * grad_scale.  When
 * param_bf16 is non-NULL it receives bf16(master) after the update.  This is
 * the step a data-parallel trainer runs on its own shard between the
 * reduce-scatter of the gradients and the all-gather of the weights.  fp32
 * buffers 16-byte aligned, param_bf16 8-byte aligned. */
int mea_adamw_step(long long n, float* master, float* exp_avg, float* exp_avg_sq, const float* grad,
                   void* param_bf16, double lr, double beta1, double beta2, double eps, double weight_decay,
                   float grad_scale, int step, void* stream);

/* ---------------------------------------------------------------- profiling
 * No counterpart in the reference (it has no timing hooks).  When enabled,
 * mea_block_forward / mea_block_backward record CUDA events on the caller's
 * stream around each of their kernels. */

/* Enables (on != 0) or disables recording and drops recorded events. */
int mea_profile_enable(int on);
/* Synchronises the recorded events, writes per-stage total milliseconds and
 * launch counts (arrays of max_stages), clears the record; returns the number
 * of stages the library knows (or a negative error). */
int mea_profile_read(int max_stages, float* total_ms, int* counts);
/* Name of a profiling stage ("" when out of range). */
const char* mea_profile_stage_name(int stage);

#ifdef __cplusplus
}
#endif

#endif /* MEA_H_ */
