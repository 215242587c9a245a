// One AdamW element update with torch.optim.AdamW semantics (decoupled
// weight decay p *= 1 - lr*wd, bias-corrected moments, eps added to the
// corrected square root), shared by the single-GPU optimizer kernel and the
// fused data-parallel reduce / update / gather kernel.
#pragma once

struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt;
};

__device__ __forceinline__ void adamw_elem(float& p, float& m, float& v, float g, bool decay, const AdamHyper& h) {
  if (decay) p *= 1.0f - h.lr * h.wd;
  m = m + (1.0f - h.beta1) * (g - m);
  v = h.beta2 * v + (1.0f - h.beta2) * g * g;
  const float denom = sqrtf(v) / h.bc2_sqrt + h.eps;
  p -= (h.lr / h.bc1) * m / denom;
}
