// llama3 RoPE arithmetic shared by the kernels that rotate q and k: K1
// (tvp_append.cu) and the Q/K/V projection with the append in its epilogue
// (tvp_project.cu).  One definition, so both compute the same bits.
#pragma once

#include "tvp_common.cuh"

namespace tvp {

// llama3-scaled inverse frequency of rotate-half pair `pair` (0..31):
// theta_0 = 500000, factor 32, low/high frequency factors 1/4, original
// context 8192.  Same calls (powf) and the same expression order as the
// reference ropeKernel (src/model/RoPe.cu:15-22), so the FP32 value is the
// reference's bit for bit under the same compiler flags (no fast-math,
// default FMA contraction).
__device__ __forceinline__ float llama3_theta(int pair) {
  float theta = 1.0f / powf(500000.0f, (2.0f * pair) / kHeadDim);
  float wavelength = 6.283185307179586f / theta;
  if (wavelength > 8192.0f) {
    theta /= 32.0f;
  } else if (wavelength >= 2048.0f) {
    float smooth = (8192.0f / wavelength - 1.0f) / 3.0f;
    theta = (1.0f - smooth) * theta / 32.0f + smooth * theta;
  }
  return theta;
}

// Rotation of one (x, y) = (d, d + 32) pair by cos/sin of angle = position *
// theta, src/model/RoPe.cu:23-27: x' = x cos - y sin, y' = x sin + y cos.
// cos and sin depend on the position and the pair only, so they are evaluated
// once per token row.  The products are fused as nvcc fuses the reference's
// expression (x' = fma(x, cos, -(y sin)), y' = fma(y, cos, x sin): all 2^20
// (position, pair) rotations of positions 0..32767 compared bit for bit with
// the reference kernel's output), written out so that the rounding does not
// depend on where the compiler finds cos and sin.
__device__ __forceinline__ void rope_rotate(__nv_bfloat16 x_i, __nv_bfloat16 y_i, float c, float s,
                                            __nv_bfloat16& x_o, __nv_bfloat16& y_o) {
  const float x = (float)x_i, y = (float)y_i;
  x_o = (__nv_bfloat16)__fmaf_rn(x, c, -__fmul_rn(y, s));
  y_o = (__nv_bfloat16)__fmaf_rn(y, c, __fmul_rn(x, s));
}

}  // namespace tvp
