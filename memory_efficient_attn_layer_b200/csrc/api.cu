// The extern "C" entry points of libmea.so (declared in include/mea.h) and
// the block-level orchestration of the forward and the memory-saving backward.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "gemm.cuh"
#include "launch.h"

namespace mea {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MEA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MEA_OK;
}

static int current_device() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

int num_sms() {
  static int cache[64] = {0};
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

bool smem_attr_set(const void* kernel, int bytes) {
  // cudaFuncSetAttribute is per device; remember (kernel, device) pairs done.
  static std::mutex mu;
  static const void* done_k[256];
  static int done_d[256];
  static int n_done = 0;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_done; ++i)
    if (done_k[i] == kernel && done_d[i] == dev) return true;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  if (n_done < 256) {
    done_k[n_done] = kernel;
    done_d[n_done] = dev;
    ++n_done;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Shapes, workspace layouts
// ---------------------------------------------------------------------------
static int pick_bn(int n) { return n % 256 == 0 ? 256 : 128; }

static int validate(const mea_block_dims* d) {
  if (!d) return set_error(MEA_ERR_INVALID_ARGUMENT, "dims is NULL");
  if (d->B <= 0 || d->T <= 0 || d->C <= 0 || d->H <= 0 || d->N <= 0)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "dims must be positive (B=%d T=%d C=%d H=%d N=%d)", d->B, d->T, d->C,
                     d->H, d->N);
  if (d->T % 128) return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "T=%d must be a multiple of 128", d->T);
  if (d->N != 32 && d->N != 64 && d->N != 128)
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "head dim N=%d must be 32, 64 or 128", d->N);
  if (d->C % 128) return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "C=%d must be a multiple of 128", d->C);
  if ((d->H * d->N) % 128) return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "H*N=%d must be a multiple of 128", d->H * d->N);
  if (d->T_max < d->T) return set_error(MEA_ERR_INVALID_ARGUMENT, "rotary tables have %d rows < T=%d", d->T_max, d->T);
  if (size_t(d->B) * d->T * d->H * d->N > (size_t(1) << 31))
    return set_error(MEA_ERR_UNSUPPORTED_SHAPE, "B*T*H*N must stay below 2^31");
  return MEA_OK;
}

static bool aligned(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

// Caller buffers of the block calls: the bf16 activations, weights and tables
// and the fp32 row statistics are read and written with 16-byte vector and
// TMA accesses, the workspace is carved at 256-byte offsets, and the bf16
// weight gradients are written 8 bytes at a time.  Checked before any device
// work is queued.
static int check_block_buffers(const void* const* b16, int n16, const void* const* b8, int n8, const char* who) {
  for (int i = 0; i < n16; ++i)
    if (!aligned(b16[i], 16))
      return set_error(MEA_ERR_ALIGNMENT, "%s: tensor argument %d is not 16-byte aligned", who, i);
  for (int i = 0; i < n8; ++i)
    if (!aligned(b8[i], 8))
      return set_error(MEA_ERR_ALIGNMENT, "%s: weight-gradient output %d is not 8-byte aligned", who, i);
  return MEA_OK;
}

struct Carve {
  size_t off = 0;
  size_t take(size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  }
};

struct FwdWs {
  size_t rx, q, k, v, gs, gated, bound, total;
};
static FwdWs fwd_layout(const mea_block_dims& d) {
  const size_t M = size_t(d.B) * d.T, HN = size_t(d.H) * d.N;
  FwdWs w;
  Carve c;
  w.rx = c.take(M * 4);
  w.q = c.take(M * HN * 2);
  w.k = c.take(M * HN * 2);
  w.v = c.take(M * HN * 2);
  w.gs = c.take(M * HN * 2);
  w.gated = c.take(M * HN * 2);
  w.bound = c.take(4);
  w.total = c.off;
  return w;
}

struct BwdWs {
  size_t rx, q, k, v, gs, rq, rk, gated, o, dO, delta, dacc, dqacc, dk, dxn, dw32, total;
};
// Slots are shared between tensors whose lifetimes do not overlap (kernel
// order of mea_block_backward_ex): gated is last read by the dWo GEMM and dK is
// first written by the attention backward, after it; sigmoid(g) is last read by
// the gate backward, whose epilogue writes dO over it (each warp loads a head's
// sigmoid(g) rows before it stores that head's dO rows at the same positions,
// and no other tile reads them).
// The projection gradient dAcc = [dq | dk | dv | dg] (one row per token):
//  * head dim >= 64: no buffer of its own.  Each part is written over the
//    tensor its producer consumes last, in the same [B,H,T,N] layout: dg over
//    O (gate backward epilogue, as dO over sigmoid(g)); dv over v (attention
//    backward: V tile j is read only by the work item that writes dV tile j,
//    before it writes it); dq, dk over q, k (q/k backward: each element is read
//    by the thread that then writes it).  The dW and dx GEMMs read the four
//    parts per head (A_MN_HEADS / A_K_HEADS), and dx_n goes to the gated/dK
//    slot or the dQ accumulator's, both dead by then.
//  * head dim 32 (a 64-wide GEMM box spans two heads): one [M, 4*H*N] buffer;
//    dx_n takes O's slot (O is last read by the gate backward).
static bool dacc_in_place(const mea_block_dims& d) { return d.N >= 64; }

static BwdWs bwd_layout(const mea_block_dims& d) {
  const size_t M = size_t(d.B) * d.T, HN = size_t(d.H) * d.N, BHT = size_t(d.B) * d.H * d.T;
  const bool inplace = dacc_in_place(d);
  BwdWs w;
  Carve c;
  w.rx = c.take(M * 4);
  w.q = c.take(M * HN * 2);
  w.k = c.take(M * HN * 2);
  w.v = c.take(M * HN * 2);
  w.gs = c.take(M * HN * 2);
  w.rq = c.take(BHT * 4);
  w.rk = c.take(BHT * 4);
  w.gated = c.take(M * HN * 2);
  w.o = c.take(M * HN * 2);
  w.dO = w.gs;
  w.delta = c.take(BHT * 4);
  w.dacc = inplace ? 0 : c.take(M * 4 * HN * 2);
  w.dqacc = c.take(M * HN * 4);
  w.dk = w.gated;
  // gated / O slots hold [M, H*N] bf16, the dQ accumulator [M, H*N] fp32; dx_n is [M, C] bf16
  if (inplace)
    w.dxn = size_t(d.C) <= HN ? w.gated : size_t(d.C) <= 2 * HN ? w.dqacc : c.take(M * d.C * 2);
  else
    w.dxn = size_t(d.C) <= HN ? w.o : c.take(M * d.C * 2);
  w.dw32 = c.take(5 * HN * d.C * 4);
  w.total = c.off;
  return w;
}

// ---------------------------------------------------------------------------
// Building blocks
// ---------------------------------------------------------------------------
// Fused q/k/v/g projection.  `a` is x_n, or x itself with `row_scale` = the
// input RMSNorm's inverse RMS per row (the norm applied to the accumulator rows
// in the epilogue: x_n W^T = diag(r) x W^T).
static int qkvg(const mea_block_dims& d, const void* a, const float* row_scale, const void* wq, const void* wk,
                const void* wv, const void* wg, const void* f1, const void* f2, void* q, void* k, void* v, void* gs,
                float* rq, float* rk, int* status, cudaStream_t st) {
  const int HN = d.H * d.N;
  GemmLaunch L{};
  L.M = d.B * d.T;
  L.N = 4 * HN;
  L.K = d.C;
  L.bn = 256;
  L.amode = A_K;
  L.bmode = B_SLABS;
  L.epi = EPI_QKVG;
  L.a = a;
  L.lda = d.C;
  L.b[0] = wq;
  L.b[1] = wk;
  L.b[2] = wv;
  L.b[3] = wg;
  L.ldb = d.C;
  L.b_rows = HN;
  L.slab_rows = d.N;
  L.k_splits = 1;
  GemmParams p{};
  p.status = status;
  L.out[0] = q;
  L.out[1] = k;
  L.out[2] = v;
  L.out[3] = gs;
  L.in[0] = f1;
  L.in[1] = f2;
  L.ldin = d.N;
  L.in_rows = d.T_max;
  p.rq = rq;
  p.rk = rk;
  p.row_scale = row_scale;
  p.T = d.T;
  p.H = d.H;
  p.hd = d.N;
  p.eps = d.eps;
  return run_gemm(L, p, st);
}

// `row_scale` (may be NULL) multiplies each row of dg_pre; `dg_heads`: dg is
// [B,H,T,N] (ld_dg unused), else [M, ld_dg] with head h at column h*N.
static int gate_bwd(const mea_block_dims& d, const void* dy, const void* wo, const void* o, const void* gs, void* dO,
                    void* dg, long long ld_dg, float* delta, const float* row_scale, bool dg_heads, int* status,
                    cudaStream_t st) {
  const int HN = d.H * d.N;
  GemmLaunch L{};
  L.M = d.B * d.T;
  L.N = HN;
  L.K = d.C;
  L.bn = pick_bn(HN);
  L.amode = A_K;
  L.bmode = B_MN;
  L.epi = EPI_DGATE;
  L.a = dy;
  L.lda = d.C;
  L.b[0] = wo;
  L.ldb = HN;
  L.k_splits = 1;
  GemmParams p{};
  p.status = status;
  L.in[0] = o;
  L.in[1] = gs;
  L.out[0] = dO;
  L.out[1] = dg;
  L.ldo = ld_dg;
  p.delta = delta;
  p.row_scale = row_scale;
  p.dg_heads = dg_heads ? 1 : 0;
  p.T = d.T;
  p.H = d.H;
  p.hd = d.N;
  return run_gemm(L, p, st);
}

// Split-K weight-gradient GEMM: out[M', N'] += A^T B over the token dim.  With
// `a_parts` (and `d`), A^T is the four per-head dAcc parts (M' = 4*H*N).
static int weight_grad(int Mp, int Np, int tokens, const void* a, long long lda, const void* b, long long ldb,
                       float* out, int* status, cudaStream_t st, const void* const* a_parts = nullptr,
                       const mea_block_dims* d = nullptr) {
  GemmLaunch L{};
  L.M = Mp;
  L.N = Np;
  L.K = tokens;
  L.bn = pick_bn(Np);
  L.amode = a_parts ? A_MN_HEADS : A_MN;
  L.bmode = B_MN;
  L.epi = EPI_RED_F32;
  L.a = a;
  L.lda = lda;
  L.b[0] = b;
  L.ldb = ldb;
  L.k_splits = auto_splits(Mp / GEMM_BM, Np / L.bn, tokens / GEMM_BK, 8);
  GemmParams p{};
  p.status = status;
  if (a_parts) {
    for (int i = 0; i < 4; ++i) L.a4[i] = a_parts[i];
    p.H = d->H;
    p.T = d->T;
    p.hd = d->N;
  }
  L.out[0] = out;
  L.ldo = Np;
  return run_gemm(L, p, st);
}


// ---------------------------------------------------------------------------
// Optional per-stage timing: CUDA events recorded on the caller's stream around
// every kernel of the block calls (mea_profile_enable / mea_profile_read).
// ---------------------------------------------------------------------------
enum Stage : int {
  ST_FWD_NORM = 0, ST_FWD_QKVG, ST_FWD_ATTN, ST_FWD_OPROJ,
  ST_BWD_NORM, ST_BWD_QKVG, ST_BWD_ATTN_FWD, ST_BWD_MEMSET, ST_BWD_DWO, ST_BWD_DGATE, ST_BWD_ATTN, ST_BWD_QK,
  ST_BWD_DW, ST_BWD_DX, ST_BWD_NORM_BWD, ST_BWD_CAST, ST_BWD_GATE_REPACK, ST_COUNT
};
static const char* kStageNames[ST_COUNT] = {
  "fwd.rmsnorm", "fwd.qkvg_gemm", "fwd.attention", "fwd.o_proj_gemm",
  "bwd.rmsnorm", "bwd.qkvg_gemm", "bwd.attention_recompute", "bwd.memset", "bwd.dWo_gemm", "bwd.dgate_gemm",
  "bwd.attention_bwd", "bwd.qk_norm_rope_bwd", "bwd.dW_gemm", "bwd.dx_gemm", "bwd.rmsnorm_bwd", "bwd.cast",
  "bwd.gate_repack"};

struct Profiler {
  std::mutex mu;
  bool on = false;
  struct Rec { int stage; cudaEvent_t a, b; };
  std::vector<Rec> recs;
  std::vector<cudaEvent_t> pool;
  cudaEvent_t get() {
    if (!pool.empty()) { cudaEvent_t e = pool.back(); pool.pop_back(); return e; }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
};
static Profiler g_prof;

struct StageScope {
  int stage;
  cudaStream_t st;
  cudaEvent_t b = nullptr;
  StageScope(int s, cudaStream_t stream) : stage(s), st(stream) {
    if (!g_prof.on) return;
    std::lock_guard<std::mutex> lock(g_prof.mu);
    cudaEvent_t a = g_prof.get();
    b = g_prof.get();
    cudaEventRecord(a, st);
    g_prof.recs.push_back({stage, a, b});
  }
  ~StageScope() {
    if (b) cudaEventRecord(b, st);
  }
};

#define MEA_TRY(expr)            \
  do {                           \
    const int rc_ = (expr);      \
    if (rc_ != MEA_OK) return rc_; \
  } while (0)

#define MEA_STAGE(id, expr)        \
  do {                             \
    StageScope scope_(id, st);     \
    MEA_TRY(expr);                 \
  } while (0)

static int record_event(void* ev, cudaStream_t st) {
  if (!ev) return MEA_OK;
  if (cudaEventRecord(static_cast<cudaEvent_t>(ev), st) != cudaSuccess)
    return set_error(MEA_ERR_CUDA, "cudaEventRecord failed: %s", cudaGetErrorString(cudaGetLastError()));
  return MEA_OK;
}

static int memset_async(void* p, size_t bytes, cudaStream_t st) {
  if (!p || !bytes) return MEA_OK;
  if (cudaMemsetAsync(p, 0, bytes, st) != cudaSuccess) return set_error(MEA_ERR_CUDA, "cudaMemsetAsync failed");
  return MEA_OK;
}

}  // namespace mea

using namespace mea;

extern "C" {

int mea_version(void) { return 100; }

const char* mea_last_error_string(void) { return g_err; }

int mea_device_check(void) {
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, current_device()) != cudaSuccess)
    return set_error(MEA_ERR_CUDA, "cudaGetDeviceProperties failed");
  if (prop.major != 10 || prop.minor != 0)
    return set_error(MEA_ERR_UNSUPPORTED_DEVICE, "device is sm_%d%d; libmea is built for sm_100a only", prop.major,
                     prop.minor);
  return MEA_OK;
}

int mea_read_status(const int* status_dev, int* out, void* stream) {
  if (!status_dev || !out) return set_error(MEA_ERR_INVALID_ARGUMENT, "status pointers are NULL");
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return set_error(MEA_ERR_CUDA, "stream sync: %s", cudaGetErrorString(cudaGetLastError()));
  if (cudaMemcpy(out, status_dev, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return set_error(MEA_ERR_CUDA, "status copy failed");
  if (*out != 0)
    return set_error(MEA_ERR_DEVICE_TIMEOUT, "device wait timed out (kernel %d, site %d)", (*out >> 8) & 0xFF,
                     (*out >> 16) & 0xFFFF);
  return MEA_OK;
}

size_t mea_forward_workspace_size(const mea_block_dims* d) {
  if (validate(d) != MEA_OK) return 0;
  return fwd_layout(*d).total;
}

size_t mea_backward_workspace_size(const mea_block_dims* d) {
  if (validate(d) != MEA_OK) return 0;
  return bwd_layout(*d).total;
}

static int block_forward(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                         const void* wg, const void* wo, const void* factor1, const void* factor2, void* y,
                         float* lse2, void* o_out, void* workspace, size_t workspace_bytes, int* status, void* stream) {
  MEA_TRY(validate(d));
  const FwdWs w = fwd_layout(*d);
  if (!workspace || workspace_bytes < w.total)
    return set_error(MEA_ERR_WORKSPACE, "forward workspace needs %zu bytes, got %zu", w.total, workspace_bytes);
  if (!x || !wq || !wk || !wv || !wg || !wo || !factor1 || !factor2 || !y || !lse2)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "forward: NULL tensor pointer");
  {
    const void* b16[] = {x, wq, wk, wv, wg, wo, factor1, factor2, y, lse2, o_out};
    MEA_TRY(check_block_buffers(b16, 11, nullptr, 0, "forward"));
    if (!aligned(workspace, 256)) return set_error(MEA_ERR_ALIGNMENT, "forward: workspace must be 256-byte aligned");
  }
  auto st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const int M = d->B * d->T, HN = d->H * d->N;
  // Input RMSNorm fused into the projection: only the inverse RMS per row is
  // computed here; the GEMM runs on x and scales its accumulator rows.
  float* rx = reinterpret_cast<float*>(ws + w.rx);
  MEA_STAGE(ST_FWD_NORM, run_rmsnorm_fwd(M, d->C, d->eps, x, nullptr, rx, st));
  MEA_STAGE(ST_FWD_QKVG, qkvg(*d, x, rx, wq, wk, wv, wg, factor1, factor2, ws + w.q, ws + w.k, ws + w.v, ws + w.gs, nullptr,
               nullptr, status, st));
  {
    // Scores are bounded through the per-head norm and the rotary tables, so
    // the attention uses that bound as its exp2 reference (no row-max pass).
    StageScope scope_(ST_FWD_ATTN, st);
    float* bound = reinterpret_cast<float*>(ws + w.bound);
    MEA_TRY(run_rope_bound(d->T, d->N, factor1, factor2, d->N, bound, st));
    MEA_TRY(run_attn_fwd(d->B, d->H, d->T, d->N, ws + w.q, ws + w.k, ws + w.v, ws + w.gs, ws + w.gated, lse2, o_out,
                         bound, nullptr, status, st));
  }
  GemmLaunch L{};
  L.M = M;
  L.N = d->C;
  L.K = HN;
  L.bn = pick_bn(d->C);
  L.amode = A_K;
  L.bmode = B_K;
  L.epi = EPI_BF16;
  L.a = ws + w.gated;
  L.lda = HN;
  L.b[0] = wo;
  L.ldb = HN;
  L.k_splits = 1;
  L.out[0] = y;
  L.ldo = d->C;
  GemmParams p{};
  p.status = status;
  StageScope scope_(ST_FWD_OPROJ, st);
  return run_gemm(L, p, st);
}

int mea_block_forward(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                      const void* wg, const void* wo, const void* factor1, const void* factor2, void* y, float* lse2,
                      void* workspace, size_t workspace_bytes, int* status, void* stream) {
  return block_forward(d, x, wq, wk, wv, wg, wo, factor1, factor2, y, lse2, nullptr, workspace, workspace_bytes,
                       status, stream);
}

int mea_block_forward_save_o(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                             const void* wg, const void* wo, const void* factor1, const void* factor2, void* y,
                             float* lse2, void* o, void* workspace, size_t workspace_bytes, int* status,
                             void* stream) {
  if (!o) return set_error(MEA_ERR_INVALID_ARGUMENT, "forward: o is NULL");
  return block_forward(d, x, wq, wk, wv, wg, wo, factor1, factor2, y, lse2, o, workspace, workspace_bytes, status,
                       stream);
}

int mea_block_backward(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                       const void* wg, const void* wo, const void* factor1, const void* factor2, const float* lse2,
                       const void* dy, void* dx, void* dwq, void* dwk, void* dwv, void* dwg, void* dwo,
                       float* dfactor1, float* dfactor2, float* dweights_f32, void* workspace,
                       size_t workspace_bytes, int* status, void* stream) {
  return mea_block_backward_ex(d, x, wq, wk, wv, wg, wo, factor1, factor2, lse2, dy, dx, dwq, dwk, dwv, dwg, dwo,
                               dfactor1, dfactor2, dweights_f32, workspace, workspace_bytes, status, stream, nullptr,
                               nullptr);
}

// The block backward.  `o_saved` (may be NULL): the forward's attention output
// O [B,H,T,N]; when given, the attention recompute is skipped and the gated
// tile the dWo GEMM needs is formed from it.
static int block_backward(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                          const void* wg, const void* wo, const void* factor1, const void* factor2,
                          const float* lse2, const void* o_saved, const void* dy, void* dx, void* dwq, void* dwk,
                          void* dwv, void* dwg, void* dwo, float* dfactor1, float* dfactor2, float* dweights_f32,
                          void* workspace, size_t workspace_bytes, int* status, void* stream, void* ev_dwo_ready,
                          void* ev_dw_ready) {
  MEA_TRY(validate(d));
  const bool want_bf16 = dwq || dwk || dwv || dwg || dwo;
  if (!want_bf16 && !dweights_f32)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "backward: no weight-gradient output (bf16 or fp32) given");
  const BwdWs w = bwd_layout(*d);
  if (!workspace || workspace_bytes < w.total)
    return set_error(MEA_ERR_WORKSPACE, "backward workspace needs %zu bytes, got %zu", w.total, workspace_bytes);
  if (!x || !wq || !wk || !wv || !wg || !wo || !factor1 || !factor2 || !lse2 || !dy || !dx)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "backward: NULL tensor pointer");
  if ((dfactor1 == nullptr) != (dfactor2 == nullptr))
    return set_error(MEA_ERR_INVALID_ARGUMENT, "backward: dfactor1 and dfactor2 must both be set or both be NULL");
  {
    const void* b16[] = {x, wq, wk, wv, wg, wo, factor1, factor2, lse2, dy, dx, dweights_f32, o_saved};
    const void* b8[] = {dwq, dwk, dwv, dwg, dwo};
    MEA_TRY(check_block_buffers(b16, 13, b8, 5, "backward"));
    if (!aligned(workspace, 256)) return set_error(MEA_ERR_ALIGNMENT, "backward: workspace must be 256-byte aligned");
  }
  auto st = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  const int M = d->B * d->T, HN = d->H * d->N, C = d->C;
  const size_t BHTN = size_t(M) * HN;
  float* rx = reinterpret_cast<float*>(ws + w.rx);
  float* rq = reinterpret_cast<float*>(ws + w.rq);
  float* rk = reinterpret_cast<float*>(ws + w.rk);
  float* delta = reinterpret_cast<float*>(ws + w.delta);
  float* dqacc = reinterpret_cast<float*>(ws + w.dqacc);
  float* dw32 = dweights_f32 ? dweights_f32 : reinterpret_cast<float*>(ws + w.dw32);
  float* dwo32 = dw32 + size_t(4) * HN * C;
  char* dacc = dacc_in_place(*d) ? nullptr : ws + w.dacc;
  const long long ld_dacc = 4LL * HN;

  // Recompute: input norm (r only), projections (+ inverse RMS of q/k), attention (+ O).
  MEA_STAGE(ST_BWD_NORM, run_rmsnorm_fwd(M, C, d->eps, x, nullptr, rx, st));
  // Same projection as the forward (x with the row scale), so the recomputed
  // q/k/v/g match the forward's bit for bit and the saved LSE stays exact.
  // x_n itself is never stored: every writer of dAcc multiplies row m by r_m
  // (dAcc' = diag(r) dAcc: the gate backward's epilogue, the attention
  // backward's dV read-out, and the q/k backward through rq, rk, which this
  // projection stores as r_q * r and r_k * r), so the weight gradient
  // dAcc^T x_n = dAcc'^T x and the dx GEMM yields diag(r) dx_n, which the norm
  // backward takes as is.
  MEA_STAGE(ST_BWD_QKVG, qkvg(*d, x, rx, wq, wk, wv, wg, factor1, factor2, ws + w.q, ws + w.k, ws + w.v, ws + w.gs, rq, rk,
               status, st));
  // The recompute takes the forward's LSE as its exp2 reference: P comes out
  // normalised, the same P the attention backward rebuilds.
  // (N <= 64: the recompute also clears the dQ accumulator; otherwise a memset does.)
  // With the forward's O kept, only the gated tile is formed from it.
  const bool zero_in_fwd = d->N <= 64 && !o_saved;
  const void* o = o_saved ? o_saved : ws + w.o;
  if (o_saved)
    MEA_STAGE(ST_BWD_GATE_REPACK, run_gate_repack(d->B, d->H, d->T, d->N, o_saved, ws + w.gs, ws + w.gated, st));
  else
    MEA_STAGE(ST_BWD_ATTN_FWD, run_attn_fwd(d->B, d->H, d->T, d->N, ws + w.q, ws + w.k, ws + w.v, ws + w.gs,
                                            ws + w.gated, nullptr, ws + w.o, nullptr, lse2, status, st,
                                            zero_in_fwd ? dqacc : nullptr));
  {
    StageScope scope_(ST_BWD_MEMSET, st);
    MEA_TRY(memset_async(dw32, size_t(5) * HN * C * 4, st));
    if (!zero_in_fwd) MEA_TRY(memset_async(dqacc, BHTN * 4, st));
    MEA_TRY(memset_async(dfactor1, size_t(d->T_max) * d->N * 4, st));
    MEA_TRY(memset_async(dfactor2, size_t(d->T_max) * d->N * 4, st));
  }
  // o_proj backward: dWo = dY^T gated; dGated = dY Wo with the gate backward fused.
  MEA_STAGE(ST_BWD_DWO, weight_grad(C, HN, M, dy, C, ws + w.gated, HN, dwo32, status, st));
  MEA_TRY(record_event(ev_dwo_ready, st));
  // dAcc parts: in place over O, v, q, k (per-head layout), or the dacc buffer.
  const bool inplace = dacc_in_place(*d);
  const void* parts[4] = {ws + w.q, ws + w.k, ws + w.v, ws + w.o};
  MEA_STAGE(ST_BWD_DGATE, gate_bwd(*d, dy, wo, o, ws + w.gs, ws + w.dO,
                                   inplace ? ws + w.o : dacc + size_t(3) * HN * 2, ld_dacc, delta, rx, inplace,
                                   status, st));
  // Attention backward: dq (fp32 accumulate), dk, dv (over v, or the v part of dacc).
  MEA_STAGE(ST_BWD_ATTN, run_attn_bwd(d->B, d->H, d->T, d->N, ws + w.q, ws + w.k, ws + w.v, ws + w.dO, lse2, delta,
                                      dqacc, ws + w.dk, inplace ? ws + w.v : dacc + size_t(2) * HN * 2, ld_dacc,
                                      status, st, rx, inplace));
  // q/k norm + rotary backward -> dq, dk of dAcc; rotary-table gradients.
  if (inplace)
    MEA_STAGE(ST_BWD_QK, run_qk_norm_rope_bwd_inplace(d->B, d->H, d->T, d->N, dqacc, ws + w.dk, ws + w.q, ws + w.k,
                                                      rq, rk, factor1, factor2, d->N, dfactor1, dfactor2, st));
  else
    MEA_STAGE(ST_BWD_QK, run_qk_norm_rope_bwd(d->B, d->H, d->T, d->N, dqacc, ws + w.dk, ws + w.q, ws + w.k, rq, rk,
                                              factor1, factor2, d->N, dacc, ld_dacc, dfactor1, dfactor2, st));
  // Projection weight gradients: [4HN, C] = dacc^T xn = (diag(r) dacc)^T x.
  MEA_STAGE(ST_BWD_DW, weight_grad(4 * HN, C, M, dacc, ld_dacc, x, C, dw32, status, st, inplace ? parts : nullptr, d));
  MEA_TRY(record_event(ev_dw_ready, st));
  // diag(r) dx_normed = (diag(r) dacc) [Wq; Wk; Wv; Wg]
  {
    GemmLaunch L{};
    L.M = M;
    L.N = C;
    L.K = 4 * HN;
    L.bn = pick_bn(C);
    L.amode = inplace ? A_K_HEADS : A_K;
    L.bmode = B_MN_KSPLIT4;
    L.epi = EPI_BF16;
    L.a = dacc;
    L.lda = ld_dacc;
    for (int i = 0; i < 4; ++i) L.a4[i] = parts[i];
    L.b[0] = wq;
    L.b[1] = wk;
    L.b[2] = wv;
    L.b[3] = wg;
    L.ldb = C;
    L.b_rows = HN;
    L.k_splits = 1;
    L.out[0] = ws + w.dxn;
    L.ldo = C;
    GemmParams p{};
    p.status = status;
    p.H = d->H;
    p.T = d->T;
    p.hd = d->N;
    MEA_STAGE(ST_BWD_DX, run_gemm(L, p, st));
  }
  MEA_STAGE(ST_BWD_NORM_BWD, run_rmsnorm_bwd(M, C, ws + w.dxn, x, rx, dx, st, /*prescaled=*/true));
  const size_t wsz = size_t(HN) * C;
  StageScope cast_scope(ST_BWD_CAST, st);
  void* dst[5] = {dwq, dwk, dwv, dwg, dwo};
  MEA_TRY(run_cast_f32_bf16_parts((long long)wsz, dw32, dst, 5, st));
  return MEA_OK;
}

int mea_block_backward_ex(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                          const void* wg, const void* wo, const void* factor1, const void* factor2,
                          const float* lse2, const void* dy, void* dx, void* dwq, void* dwk, void* dwv, void* dwg,
                          void* dwo, float* dfactor1, float* dfactor2, float* dweights_f32, void* workspace,
                          size_t workspace_bytes, int* status, void* stream, void* ev_dwo_ready,
                          void* ev_dw_ready) {
  return block_backward(d, x, wq, wk, wv, wg, wo, factor1, factor2, lse2, nullptr, dy, dx, dwq, dwk, dwv, dwg, dwo,
                        dfactor1, dfactor2, dweights_f32, workspace, workspace_bytes, status, stream, ev_dwo_ready,
                        ev_dw_ready);
}

int mea_block_backward_from_o(const mea_block_dims* d, const void* x, const void* wq, const void* wk, const void* wv,
                              const void* wg, const void* wo, const void* factor1, const void* factor2,
                              const float* lse2, const void* o, const void* dy, void* dx, void* dwq, void* dwk,
                              void* dwv, void* dwg, void* dwo, float* dfactor1, float* dfactor2,
                              float* dweights_f32, void* workspace, size_t workspace_bytes, int* status,
                              void* stream, void* ev_dwo_ready, void* ev_dw_ready) {
  if (!o) return set_error(MEA_ERR_INVALID_ARGUMENT, "backward: o is NULL");
  return block_backward(d, x, wq, wk, wv, wg, wo, factor1, factor2, lse2, o, dy, dx, dwq, dwk, dwv, dwg, dwo,
                        dfactor1, dfactor2, dweights_f32, workspace, workspace_bytes, status, stream, ev_dwo_ready,
                        ev_dw_ready);
}

int mea_rmsnorm_forward(int rows, int C, float eps, const void* x, void* xn, float* r, void* stream) {
  return run_rmsnorm_fwd(rows, C, eps, x, xn, r, static_cast<cudaStream_t>(stream));
}

int mea_qkvg_forward(const mea_block_dims* d, const void* xn, const void* wq, const void* wk, const void* wv,
                     const void* wg, const void* factor1, const void* factor2, void* q, void* k, void* v, void* gs,
                     float* rq, float* rk, int* status, void* stream) {
  MEA_TRY(validate(d));
  return qkvg(*d, xn, nullptr, wq, wk, wv, wg, factor1, factor2, q, k, v, gs, rq, rk, status,
              static_cast<cudaStream_t>(stream));
}

int mea_attention_forward(int B, int H, int T, int N, const void* q, const void* k, const void* v, const void* gs,
                          void* gated, float* lse2, void* o, int* status, void* stream) {
  return run_attn_fwd(B, H, T, N, q, k, v, gs, gated, lse2, o, nullptr, nullptr, status, static_cast<cudaStream_t>(stream));
}

int mea_gemm(int M, int N, int K, const void* a, long long lda, int a_mn, const void* b, long long ldb, int b_mn,
             float* out, long long ldo, int accumulate, int* status, void* stream) {
  GemmLaunch L{};
  L.M = M;
  L.N = N;
  L.K = K;
  L.bn = pick_bn(N);
  L.amode = a_mn ? A_MN : A_K;
  L.bmode = b_mn ? B_MN : B_K;
  L.epi = accumulate ? EPI_RED_F32 : EPI_F32;
  L.a = a;
  L.lda = lda;
  L.b[0] = b;
  L.ldb = ldb;
  L.k_splits = 1;
  if (accumulate && M % GEMM_BM == 0 && N % L.bn == 0 && K % GEMM_BK == 0)
    L.k_splits = auto_splits(M / GEMM_BM, N / L.bn, K / GEMM_BK, 8);
  if (accumulate && L.amode != A_MN) L.k_splits = 1;  // the reducing epilogue is built for A_MN x B_MN only
  if (accumulate && (L.amode != A_MN || L.bmode != B_MN))
    return set_error(MEA_ERR_INVALID_ARGUMENT, "mea_gemm: accumulate needs a_mn = b_mn = 1");
  L.out[0] = out;
  L.ldo = ldo;
  GemmParams p{};
  p.status = status;
  return run_gemm(L, p, static_cast<cudaStream_t>(stream));
}

int mea_gemm_e4m3(int M, int N, int K, const void* a, long long lda, const void* b, long long ldb, void* out,
                  long long ldo, int out_bf16, int* status, void* stream) {
  if (!a || !b || !out) return set_error(MEA_ERR_INVALID_ARGUMENT, "mea_gemm_e4m3: NULL operand");
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(out)) & 15 ||
      lda % 16 || ldb % 16 || ldo % (out_bf16 ? 8 : 4))
    return set_error(MEA_ERR_ALIGNMENT, "mea_gemm_e4m3: operands 16-byte aligned with 16-byte row pitches");
  GemmLaunch L{};
  L.M = M;
  L.N = N;
  L.K = K;
  L.bn = pick_bn(N);
  L.amode = A_K;
  L.bmode = B_K;
  L.epi = out_bf16 ? EPI_BF16 : EPI_F32;
  L.e4m3 = true;
  L.a = a;
  L.lda = lda;
  L.b[0] = b;
  L.ldb = ldb;
  L.k_splits = 1;
  L.out[0] = out;
  L.ldo = ldo;
  GemmParams p{};
  p.status = status;
  return run_gemm(L, p, static_cast<cudaStream_t>(stream));
}

int mea_gate_backward(const mea_block_dims* d, const void* dy, const void* wo, const void* o, const void* gs,
                      void* dO, void* dg, long long ld_dg, float* delta, int* status, void* stream) {
  MEA_TRY(validate(d));
  return gate_bwd(*d, dy, wo, o, gs, dO, dg, ld_dg, delta, nullptr, false, status, static_cast<cudaStream_t>(stream));
}

int mea_attention_backward(int B, int H, int T, int N, const void* q, const void* k, const void* v, const void* dO,
                           const float* lse2, const float* delta, float* dq_acc, void* dk, void* dv, long long ld_dv,
                           int* status, void* stream) {
  return run_attn_bwd(B, H, T, N, q, k, v, dO, lse2, delta, dq_acc, dk, dv, ld_dv, status,
                      static_cast<cudaStream_t>(stream));
}

int mea_qk_norm_rope_backward(const mea_block_dims* d, const float* dq_acc, const void* dk, const void* q,
                              const void* k, const float* rq, const float* rk, const void* factor1,
                              const void* factor2, void* dacc, long long ld_dacc, float* dfactor1, float* dfactor2,
                              void* stream) {
  MEA_TRY(validate(d));
  if ((dfactor1 == nullptr) != (dfactor2 == nullptr))
    return set_error(MEA_ERR_INVALID_ARGUMENT, "dfactor1 and dfactor2 must both be set or both be NULL");
  return run_qk_norm_rope_bwd(d->B, d->H, d->T, d->N, dq_acc, dk, q, k, rq, rk, factor1, factor2, d->N, dacc, ld_dacc,
                              dfactor1, dfactor2, static_cast<cudaStream_t>(stream));
}

int mea_rmsnorm_backward(int rows, int C, const void* dxn, const void* x, const float* r, void* dx, void* stream) {
  return run_rmsnorm_bwd(rows, C, dxn, x, r, dx, static_cast<cudaStream_t>(stream));
}

int mea_adamw_step(long long n, float* master, float* exp_avg, float* exp_avg_sq, const float* grad,
                   void* param_bf16, double lr, double beta1, double beta2, double eps, double weight_decay,
                   float grad_scale, int step, void* stream) {
  return run_adamw(n, master, exp_avg, exp_avg_sq, grad, param_bf16, lr, beta1, beta2, eps, weight_decay, grad_scale,
                   step, static_cast<cudaStream_t>(stream));
}

int mea_profile_enable(int on) {
  std::lock_guard<std::mutex> lock(g_prof.mu);
  for (auto& r : g_prof.recs) {
    g_prof.pool.push_back(r.a);
    g_prof.pool.push_back(r.b);
  }
  g_prof.recs.clear();
  g_prof.on = on != 0;
  return MEA_OK;
}

int mea_profile_read(int max_stages, float* total_ms, int* counts) {
  if (!total_ms || !counts || max_stages <= 0) return set_error(MEA_ERR_INVALID_ARGUMENT, "profile buffers are NULL");
  std::lock_guard<std::mutex> lock(g_prof.mu);
  for (int i = 0; i < max_stages; ++i) {
    total_ms[i] = 0.f;
    counts[i] = 0;
  }
  for (auto& r : g_prof.recs) {
    if (cudaEventSynchronize(r.b) != cudaSuccess) return set_error(MEA_ERR_CUDA, "profile event sync failed");
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    if (r.stage < max_stages) {
      total_ms[r.stage] += ms;
      counts[r.stage] += 1;
    }
    g_prof.pool.push_back(r.a);
    g_prof.pool.push_back(r.b);
  }
  g_prof.recs.clear();
  return ST_COUNT;
}

const char* mea_profile_stage_name(int stage) {
  return (stage >= 0 && stage < ST_COUNT) ? kStageNames[stage] : "";
}

}  // extern "C"
