// Host-side helpers shared by the kernels' launch code: error reporting, the
// SM count, and the internal (C++) launch functions behind the C-ABI.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "mea.h"

namespace mea {

// Records a formatted message as this thread's last error; returns `code`.
int set_error(int code, const char* fmt, ...);
// Returns MEA_OK, or MEA_ERR_CUDA with the launch error recorded.
int check_launch(const char* what);
// SM count of the current device (cached per device).
int num_sms();
// Sets the dynamic shared-memory limit of `kernel` once per device.
bool smem_attr_set(const void* kernel, int bytes);

// ---- tcgen05 GEMM (gemm.cu) ----
struct GemmParams;
struct GemmLaunch {
  int M, N, K;
  int bn;      // 128 or 256
  int amode;   // A_K / A_MN / A_K_HEADS / A_MN_HEADS
  int bmode;   // B_K / B_MN / B_SLABS / B_MN_KSPLIT4
  int epi;     // EpiMode
  const void* a;
  long long lda;        // elements between rows of A as stored
  const void* a4[4];    // A_K_HEADS / A_MN_HEADS: the four [tokens*H, hd] parts of A
                        // (GemmParams H, T, hd describe them)
  const void* b[4];
  long long ldb;        // elements between rows of B as stored
  int b_rows;           // B_SLABS / B_MN_KSPLIT4: rows of each B tensor
  int slab_rows;        // B_SLABS: head dim
  int k_splits;         // > 1 only with EPI_RED_F32
  // Epilogue tensors (run_gemm builds their TMA maps):
  //   EPI_BF16 / EPI_F32 / EPI_RED_F32: out[0] = D [M, N], row pitch ldo elements
  //   EPI_QKVG : out[0..3] = q, k, v, sigmoid(g) [B*H*T, hd]; in[0..1] = rotary
  //              tables [in_rows, hd] with row pitch ldin
  //   EPI_DGATE: out[0] = dO [B*H*T, hd]; out[1] = dg_pre [M, H*hd] with row
  //              pitch ldo, or [B*H*T, hd] when GemmParams.dg_heads is set;
  //              in[0..1] = O, sigmoid(g) [B*H*T, hd]
  void* out[4];
  long long ldo;
  const void* in[2];
  long long ldin;
  int in_rows;
  bool e4m3;  // A and B are e4m3 (K-major only; EPI_F32 / EPI_BF16)
};
int run_gemm(const GemmLaunch& L, GemmParams p, cudaStream_t st);
int auto_splits(int m_tiles, int n_tiles, int kb_total, int waves);

// ---- attention (attn_fwd.cu, attn_bwd.cu) ----
// Reference for the exponentials: `lse_in` (the saved row log-sum-exp; O comes
// out normalised and lse2 is not written), else `*bound` when it is at most
// ATTN_MAX_BOUND (a device scalar bounding every scaled score), else the
// online running max.  Both pointers may be NULL.  `dq_zero` (fp32 [B,H,T,N],
// may be NULL; head dim <= 64 only) is zeroed by the kernel's epilogue: the
// backward's dQ accumulator, cleared while the recompute runs.
constexpr float ATTN_MAX_BOUND = 50.f;
int run_attn_fwd(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* gs, void* gated,
                 float* lse2, void* o_out, const float* bound, const float* lse_in, int* status, cudaStream_t st,
                 float* dq_zero = nullptr);
// `dv_row_scale` ([B*T] fp32, may be NULL): dV row (b, t) is multiplied by
// dv_row_scale[b*T + t] before it is stored.  `dv_heads`: dv is [B,H,T,N] like
// dk (ld_dv ignored); it may then be v itself, since each V tile is read only
// by the work item that writes its dV tile, and only before that write.
int run_attn_bwd(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* dO,
                 const float* lse2, const float* delta, float* dq_acc, void* dk, void* dv, long long ld_dv, int* status,
                 cudaStream_t st, const float* dv_row_scale = nullptr, bool dv_heads = false);
// The shape, pointer and alignment checks of run_attn_bwd (all but dq_acc),
// with no device work: MEA_OK or the error run_attn_bwd would return.
int check_attn_bwd_args(int B, int H, int T, int HD, const void* q, const void* k, const void* v, const void* dO,
                        const float* lse2, const float* delta, const void* dk, const void* dv, long long ld_dv);

// ---- elementwise (elementwise.cu) ----
int run_rmsnorm_fwd(int rows, int C, float eps, const void* x, void* xn, float* r, cudaStream_t st);
// `prescaled`: dxn holds r * d(x_n) (the row scale already applied upstream),
// so dx = dxn - x_n * sum(dxn * x_n) / C; otherwise dx = r * (dxn - x_n * sum(dxn * x_n) / C).
int run_rmsnorm_bwd(int rows, int C, const void* dxn, const void* x, const float* r, void* dx, cudaStream_t st,
                    bool prescaled = false);
// rq, rk: the factors from projection accumulator rows to the normalised q, k
// rows (as the fused projection stores them).
int run_qk_norm_rope_bwd(int B, int H, int T, int HD, const float* dq_acc, const void* dk, const void* q_rot,
                         const void* k_rot, const float* rq, const float* rk, const void* f1, const void* f2,
                         long long ldf, void* dacc, long long ld_dacc, float* df1, float* df2, cudaStream_t st);
// The same with the projection gradients written over q_rot / k_rot ([B,H,T,N]):
// every element is read by the thread that writes it, before it writes it.
int run_qk_norm_rope_bwd_inplace(int B, int H, int T, int HD, const float* dq_acc, const void* dk, void* q_rot,
                                 void* k_rot, const float* rq, const float* rk, const void* f1, const void* f2,
                                 long long ldf, float* df1, float* df2, cudaStream_t st);
int run_cast_f32_bf16(long long n, const float* src, void* dst, cudaStream_t st);
// gated[b,t,h*N+n] = o[b,h,t,n] * gs[b,h,t,n] (all bf16).
int run_gate_repack(int B, int H, int T, int HD, const void* o, const void* gs, void* gated, cudaStream_t st);
// `parts` (<= 5) consecutive fp32 blocks of n elements into dst[i] (NULL: skipped), one launch.
int run_cast_f32_bf16_parts(long long n, const float* src, void* const* dst, int parts, cudaStream_t st);
// *out = bound (log2 units) on every scaled score q.k/sqrt(N) of the block.
int run_rope_bound(int T, int HD, const void* f1, const void* f2, long long ldf, float* out, cudaStream_t st);

// ---- optimizer (optim.cu) ----
int run_adamw(long long n, float* master, float* exp_avg, float* exp_avg_sq, const float* grad, void* param,
              double lr, double beta1, double beta2, double eps, double weight_decay, float grad_scale, int step,
              cudaStream_t st);

}  // namespace mea
