// Activations of the reference's GEMM epilogue and GLU (app/gpu/gemm.js:24, kernels.js:346-360):
// SiLU, and the tanh approximation of GELU (PyTorch's approximate="tanh", Gemma's MLP,
// tools/reference.py:198): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).  Shared by the GLU kernel
// and the linear kernel's fused GLU epilogue, so the two forms compute the same values.
#pragma once

namespace nsa {

template <int ACT>   // 0: SiLU, 1: GELU (tanh)
__device__ __forceinline__ float glu_act(float x) {
  if constexpr (ACT == 0) {
    return x / (1.f + expf(-x));
  } else {
    return 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
  }
}

}  // namespace nsa
