// AdamW update shared by the standalone fused_adamw kernel and the landing
// kernel's streamed-optimizer op.  The update of torch.optim.AdamW
// (decoupled weight decay, bias-corrected moments), in its operation order:
//   p *= 1 - lr*wd ; m += (1-b1) (g - m) ; v = b2 v + (1-b2) g^2
//   p -= (lr / (1-b1^t)) * m / (sqrt(v) / sqrt(1-b2^t) + eps)
// Every scalar factor is formed on the host in double precision and rounded
// once to float (AdamCoeffs::make), as torch forms its Python-float scalars:
// 1 - b2 taken in float from a float b2 would be off by 1.3e-5 relative.
#pragma once

#include <cmath>
#include <cstdint>

namespace ppb {

struct AdamCoeffs {
  float decay;        // 1 - lr * weight_decay
  float beta1;
  float beta2;
  float omb1;         // 1 - beta1
  float omb2;         // 1 - beta2
  float eps;
  float grad_scale;   // multiplies the incoming gradient
  float step_size;    // lr / (1 - beta1^t)
  float sqrt_bc2;     // sqrt(1 - beta2^t)

  static AdamCoeffs make(double lr, double beta1, double beta2, double eps, double weight_decay,
                         double grad_scale, int step);
};

#ifndef __CUDA_ARCH__
inline AdamCoeffs AdamCoeffs::make(double lr, double beta1, double beta2, double eps,
                                   double weight_decay, double grad_scale, int step) {
  const double bc1 = 1.0 - std::pow(beta1, step);
  const double bc2 = 1.0 - std::pow(beta2, step);
  return AdamCoeffs{static_cast<float>(1.0 - lr * weight_decay), static_cast<float>(beta1),
                    static_cast<float>(beta2), static_cast<float>(1.0 - beta1),
                    static_cast<float>(1.0 - beta2), static_cast<float>(eps),
                    static_cast<float>(grad_scale), static_cast<float>(lr / bc1),
                    static_cast<float>(std::sqrt(bc2))};
}
#endif

#ifdef __CUDACC__
__device__ __forceinline__ float adamw_update(float& m, float& v, float master, float g,
                                              const AdamCoeffs& c) {
  const float gr = g * c.grad_scale;
  float p = master * c.decay;
  m = __fadd_rn(m, __fmul_rn(c.omb1, __fsub_rn(gr, m)));
  v = __fadd_rn(__fmul_rn(v, c.beta2), __fmul_rn(__fmul_rn(gr, gr), c.omb2));
  const float denom = __fadd_rn(__fdiv_rn(sqrtf(v), c.sqrt_bc2), c.eps);
  p = __fsub_rn(p, __fmul_rn(c.step_size, __fdiv_rn(m, denom)));
  return p;
}
#endif

}  // namespace ppb
