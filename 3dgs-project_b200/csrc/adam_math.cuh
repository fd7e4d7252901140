// adam_math.cuh - the Adam arithmetic shared by every kernel that applies an Adam step (adam.cu, dp_adam.cu and
// the preprocess backward fused with the step in gs3d_backward.cu), so that a fused step and a separate one give
// the same bits.
//
// Per element (Faster-GS's adam_step_cu, cluster/patches/fastergs_lean_adam.patch:88-130):
//   m = beta1 (m - g) + g;  v = beta2 (v - g^2) + g^2
//   p -= step_size * m / fma(sqrt(v), bc2_sqrt_rcp, eps)
// with the bias corrections of the reference's host wrapper (same patch, lines 162-164), computed in double and
// rounded once to float: step_size = lr / (1 - beta1^t), bc2_sqrt_rcp = 1 / sqrt(1 - beta2^t).
#pragma once

#include <cmath>

namespace splat {

// Every operation is rounded on its own or is an explicit fused multiply-add, so the compiler cannot contract an
// operation that produced g (a product, in the fused backward) into this arithmetic: the result depends on g's
// value only, wherever it comes from.
__device__ __forceinline__ void adam_element(float& p, float g, float& m, float& v, float step_size,
                                             float bc2_sqrt_rcp, float beta1, float beta2, float eps) {
    const float g2 = __fmul_rn(g, g);
    m = fmaf(beta1, __fsub_rn(m, g), g);
    v = fmaf(beta2, __fsub_rn(v, g2), g2);
    const float denom = fmaf(__fsqrt_rn(v), bc2_sqrt_rcp, eps);
    p = __fsub_rn(p, __fdiv_rn(__fmul_rn(step_size, m), denom));
}

inline void adam_bias_corrections(double lr, double beta1, double beta2, int step, float& step_size,
                                  float& bc2_sqrt_rcp) {
    const double bc1_rcp = 1.0 / (1.0 - std::pow(beta1, step));
    step_size = static_cast<float>(lr * bc1_rcp);
    bc2_sqrt_rcp = static_cast<float>(1.0 / std::sqrt(1.0 - std::pow(beta2, step)));
}

}  // namespace splat
