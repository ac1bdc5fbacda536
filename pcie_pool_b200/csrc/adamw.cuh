// AdamW update shared by the standalone fused_adamw kernel and the landing
// kernel's streamed-optimizer op.  Same update as torch.optim.AdamW
// (decoupled weight decay, bias-corrected moments):
//   p *= 1 - lr*wd ; m = b1 m + (1-b1) g ; v = b2 v + (1-b2) g^2
//   p -= (lr / (1-b1^t)) * m / (sqrt(v) / sqrt(1-b2^t) + eps)
// The step-dependent factors are folded on the host (AdamCoeffs).
#pragma once

#include <cstdint>

namespace ppb {

struct AdamCoeffs {
  float lr;
  float beta1;
  float beta2;
  float eps;
  float weight_decay;
  float grad_scale;     // multiplies the incoming gradient
  float step_size;      // lr / (1 - beta1^t)
  float inv_sqrt_bc2;   // 1 / sqrt(1 - beta2^t)
};

#ifdef __CUDACC__
__device__ __forceinline__ float adamw_update(float& m, float& v, float master, float g,
                                              const AdamCoeffs& c) {
  const float gr = g * c.grad_scale;
  float p = master * (1.0f - c.lr * c.weight_decay);
  m = c.beta1 * m + (1.0f - c.beta1) * gr;
  v = c.beta2 * v + (1.0f - c.beta2) * gr * gr;
  const float denom = sqrtf(v) * c.inv_sqrt_bc2 + c.eps;
  p -= c.step_size * (m / denom);
  return p;
}
#endif

}  // namespace ppb
