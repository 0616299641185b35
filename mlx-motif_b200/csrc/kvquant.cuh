// Device helpers shared by the KV-cache writers (quant.cu) and the fused decode
// attention (attention.cu): the MLX affine group quantizer and RoPE of one channel.
#pragma once

#include "common.cuh"

namespace motif {

// Quantize one group whose values are spread over LPG consecutive lanes, 8 per
// lane. Returns this lane's packed word(s) and the group's scale and bias.
template <int LPG>
__device__ __forceinline__ void quant_group(const float (&v)[8], int bits, uint32_t (&words)[2],
                                            float& scale_out, float& bias_out) {
  float mx = v[0], mn = v[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) {
    mx = fmaxf(mx, v[j]);
    mn = fminf(mn, v[j]);
  }
#pragma unroll
  for (int o = LPG / 2; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
  }
  const float n_bins = (float)((1 << bits) - 1);
  float scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), n_bins), 1e-7f);
  const bool side = fabsf(mn) > fabsf(mx);
  scale = side ? scale : -scale;
  const float edge = side ? mn : mx;
  const float q0 = roundf(__fdiv_rn(edge, scale));
  const bool at_zero = (q0 == 0.0f);
  scale = at_zero ? scale : __fdiv_rn(edge, q0);
  const float bias = at_zero ? 0.0f : edge;
  uint32_t codes[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float t = roundf(__fdiv_rn(__fsub_rn(v[j], bias), scale));
    t = fminf(fmaxf(t, 0.0f), n_bins);
    codes[j] = (uint32_t)t;
  }
  if (bits == 4) {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) w |= codes[j] << (4 * j);
    words[0] = w;
    words[1] = 0;
  } else {  // 8 bits
    words[0] = codes[0] | (codes[1] << 8) | (codes[2] << 16) | (codes[3] << 24);
    words[1] = codes[4] | (codes[5] << 8) | (codes[6] << 16) | (codes[7] << 24);
  }
  scale_out = scale;
  bias_out = bias;
}

// cos/sin of θ_k = pos·inv_freq[k] (θ rounded once in fp32).
__device__ __forceinline__ void rope_angle(int k, int pos, const float* __restrict__ inv_freq, float& cs, float& sn) {
  const float theta = __fmul_rn((float)pos, inv_freq[k]);
  sincosf(theta, &sn, &cs);
}

// Rotate channel c of a head given the cos/sin of its frequency (rotate-half pairs c, c ± half).
__device__ __forceinline__ float rope_rotate(const __half* __restrict__ src, int c, int half, float cs, float sn) {
  const int k = c < half ? c : c - half;
  const float x1 = __half2float(src[k]);
  const float x2 = __half2float(src[k + half]);
  return c < half ? __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn)) : __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
}

// Non-traditional RoPE (rotate-half; the reference calls self.rope, model.py:590-594) of
// channel c of one head at position pos: θ = pos·inv_freq[c mod half]. Every step is an
// explicitly rounded fp32 operation so the value does not depend on the call site.
__device__ __forceinline__ float rope_channel(const __half* __restrict__ src, int c, int half, int pos,
                                              const float* __restrict__ inv_freq) {
  float cs, sn;
  rope_angle(c < half ? c : c - half, pos, inv_freq, cs, sn);
  return rope_rotate(src, c, half, cs, sn);
}

}  // namespace motif
