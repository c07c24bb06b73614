// AdamW step over one contiguous shard of fp32 master weights: the update a
// data-parallel trainer runs on its own shard between the reduce-scatter of
// the gradients and the all-gather of the bf16 weights.
//
// Algorithm: Adam (Kingma & Ba, 2015) with decoupled weight decay (Loshchilov
// & Hutter, 2019), in the order torch.optim.AdamW applies it:
//   w  = w * (1 - lr * wd)
//   m  = m + (1 - b1) * (g - m)
//   v  = v * b2 + (1 - b2) * g * g
//   w  = w - (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps),  bc_i = 1 - b_i^step
// with g = grad * grad_scale (1/world for the mean over data-parallel ranks).
// One HBM pass: 16 bytes read and 12 written per element of fp32 state, plus
// the 2-byte bf16 copy of the new weight.
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "launch.h"

namespace mea {

struct AdamWConsts {
  float decay;       // 1 - lr * wd
  float one_m_b1;    // 1 - b1
  float b2;
  float one_m_b2;    // 1 - b2
  float step_size;   // lr / bc1
  float bc2_sqrt;    // sqrt(bc2)
  float eps;
  float grad_scale;
};

__device__ __forceinline__ float adamw_one(float& w, float& m, float& v, float g, const AdamWConsts& c) {
  g *= c.grad_scale;
  w *= c.decay;
  m += c.one_m_b1 * (g - m);
  v = v * c.b2 + c.one_m_b2 * (g * g);
  const float denom = sqrtf(v) / c.bc2_sqrt + c.eps;
  w -= c.step_size * (m / denom);
  return w;
}

// Grid-stride over float4 groups; the last n % 4 elements go one per thread.
__global__ void __launch_bounds__(256) adamw_kernel(long long n, float* __restrict__ master, float* __restrict__ exp_avg,
                                                    float* __restrict__ exp_avg_sq, const float* __restrict__ grad,
                                                    __nv_bfloat16* __restrict__ param, AdamWConsts c) {
  const long long n4 = n >> 2;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 w = reinterpret_cast<const float4*>(master)[i];
    float4 m = reinterpret_cast<const float4*>(exp_avg)[i];
    float4 v = reinterpret_cast<const float4*>(exp_avg_sq)[i];
    const float4 g = __ldcs(reinterpret_cast<const float4*>(grad) + i);
    adamw_one(w.x, m.x, v.x, g.x, c);
    adamw_one(w.y, m.y, v.y, g.y, c);
    adamw_one(w.z, m.z, v.z, g.z, c);
    adamw_one(w.w, m.w, v.w, g.w, c);
    reinterpret_cast<float4*>(master)[i] = w;
    reinterpret_cast<float4*>(exp_avg)[i] = m;
    reinterpret_cast<float4*>(exp_avg_sq)[i] = v;
    if (param) {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(w.x, w.y);
      const __nv_bfloat162 hi = __floats2bfloat162_rn(w.z, w.w);
      uint2 packed;
      packed.x = *reinterpret_cast<const uint32_t*>(&lo);
      packed.y = *reinterpret_cast<const uint32_t*>(&hi);
      reinterpret_cast<uint2*>(param)[i] = packed;
    }
  }
  const long long t = (n4 << 2) + (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n) {
    float w = master[t], m = exp_avg[t], v = exp_avg_sq[t];
    adamw_one(w, m, v, grad[t], c);
    master[t] = w;
    exp_avg[t] = m;
    exp_avg_sq[t] = v;
    if (param) param[t] = __float2bfloat16_rn(w);
  }
}

int run_adamw(long long n, float* master, float* exp_avg, float* exp_avg_sq, const float* grad, void* param,
              double lr, double beta1, double beta2, double eps, double weight_decay, float grad_scale, int step,
              cudaStream_t st) {
  if (n < 0) return set_error(MEA_ERR_INVALID_ARGUMENT, "adamw: n=%lld must be >= 0", n);
  if (n == 0) return MEA_OK;
  if (!master || !exp_avg || !exp_avg_sq || !grad)
    return set_error(MEA_ERR_INVALID_ARGUMENT, "adamw: master, exp_avg, exp_avg_sq and grad must be non-NULL");
  if (step < 1) return set_error(MEA_ERR_INVALID_ARGUMENT, "adamw: step=%d must be >= 1", step);
  if (!(beta1 >= 0.0 && beta1 < 1.0) || !(beta2 >= 0.0 && beta2 < 1.0))
    return set_error(MEA_ERR_INVALID_ARGUMENT, "adamw: betas (%g, %g) must lie in [0, 1)", beta1, beta2);
  if (!(lr >= 0.0) || !(eps >= 0.0) || !(weight_decay >= 0.0))
    return set_error(MEA_ERR_INVALID_ARGUMENT, "adamw: lr, eps and weight_decay must be >= 0");
  for (const void* p : {(const void*)master, (const void*)exp_avg, (const void*)exp_avg_sq, (const void*)grad})
    if (reinterpret_cast<uintptr_t>(p) % 16)
      return set_error(MEA_ERR_ALIGNMENT, "adamw: fp32 buffers must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(param) % 8)
    return set_error(MEA_ERR_ALIGNMENT, "adamw: the bf16 weights must be 8-byte aligned");
  // Scalar schedule in double, rounded to fp32 once per constant (the values
  // torch.optim.AdamW's per-tensor arithmetic receives from Python floats).
  const double bc1 = 1.0 - std::pow(beta1, double(step));
  const double bc2 = 1.0 - std::pow(beta2, double(step));
  AdamWConsts c;
  c.decay = float(1.0 - lr * weight_decay);
  c.one_m_b1 = float(1.0 - beta1);
  c.b2 = float(beta2);
  c.one_m_b2 = float(1.0 - beta2);
  c.step_size = float(lr / bc1);
  c.bc2_sqrt = float(std::sqrt(bc2));
  c.eps = float(eps);
  c.grad_scale = grad_scale;
  const int threads = 256;
  const long long want = ((n >> 2) + threads - 1) / threads;
  const long long cap = (long long)num_sms() * 8;  // 8 resident CTAs of 256 threads per SM
  const int blocks = int(std::max<long long>(1, std::min(want, cap)));
  adamw_kernel<<<blocks, threads, 0, st>>>(n, master, exp_avg, exp_avg_sq, grad,
                                           static_cast<__nv_bfloat16*>(param), c);
  return check_launch("adamw_kernel");
}

}  // namespace mea
