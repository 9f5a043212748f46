// BigVGAN anti-aliased Snake activation, fused: 2x polyphase upsample ->
// Snake -> stride-2 low-pass, one pass over x, FP32 throughout.
//
// A block owns kTile consecutive outputs of one row (row = b*C + c):
//   1. xs[j] = x[clamp(t0 - 6 + j, 0, T-1)], j < kTile + 12 (replicate pad).
//   2. hs[i] = Snake(U[u]) for u = 2 t0 - 6 + i, i < 2 kTile + 12, computed
//      in (even u, odd u) pairs from 7 neighbouring xs values:
//        U[2s]   = 2 sum_j up[2j+1] x[s+2-j],   U[2s+1] = 2 sum_j up[2j] x[s+3-j].
//      Entries with u outside [0, 2T) are then overwritten with the value at
//      the clamped index (the replicate padding in front of the low-pass).
//   3. y[t0+o] = sum_k down[k] hs[2o + k + 1]; each thread emits two outputs
//      from four 16-byte shared loads.
// This is the index algebra of ops/triton/vocoder_tiled_fir.py:20-39 and
// ops/triton/alias_free.py:7-26, evaluated once per high-rate sample.
#pragma once

#include "common.cuh"

namespace isp {

constexpr int kFirTile = 2048;
constexpr int kFirThreads = 256;

struct FirParams {
  const float* x;
  int64_t rows;
  int C;
  int64_t T;
  int64_t tiles_per_row;
  const float* up;
  const float* down;
  const float* alpha;
  const float* inv_beta;
  void* y;
  const float* smooth;
  float scale;
};

ISP_D float snake(float v, float a, float ib) {
  const float s = sinf(__fmul_rn(v, a));
  return __fadd_rn(v, __fmul_rn(ib, __fmul_rn(s, s)));
}

template <bool kInt8Out>
__global__ void __launch_bounds__(kFirThreads) fir_snake_kernel(FirParams p) {
  __shared__ float s_up[12], s_down[12];
  __shared__ __align__(16) float xs[kFirTile + 12];
  __shared__ __align__(16) float hs[2 * kFirTile + 16];

  const int64_t block = blockIdx.x;
  const int64_t row = block / p.tiles_per_row;
  const int64_t t0 = (block % p.tiles_per_row) * kFirTile;
  const int64_t T = p.T;
  const int tid = threadIdx.x;
  const int c = static_cast<int>(row % p.C);
  const float a = __ldg(p.alpha + c);
  const float ib = __ldg(p.inv_beta + c);
  if (tid < 12) {
    s_up[tid] = __ldg(p.up + tid);
    s_down[tid] = __ldg(p.down + tid);
  }

  // 1. stage the low-rate halo (replicate padding by index clamping)
  const float* xrow = p.x + row * T;
  for (int j = tid; j < kFirTile + 12; j += kFirThreads) {
    int64_t t = t0 - 6 + j;
    t = t < 0 ? 0 : (t >= T ? T - 1 : t);
    xs[j] = __ldg(xrow + t);
  }
  __syncthreads();

  // 2. high-rate samples, (even, odd) pair per step
  float up[12];
#pragma unroll
  for (int k = 0; k < 12; ++k) up[k] = s_up[k];
  for (int q = tid; q < kFirTile + 6; q += kFirThreads) {
    float w[7];
#pragma unroll
    for (int j = 0; j < 7; ++j) w[j] = xs[q + j];
    float even = 0.f, odd = 0.f;
#pragma unroll
    for (int j = 0; j < 6; ++j) {
      even = fmaf(up[2 * j + 1], w[5 - j], even);
      odd = fmaf(up[2 * j], w[6 - j], odd);
    }
    float2 h;
    h.x = snake(__fmul_rn(2.f, even), a, ib);
    h.y = snake(__fmul_rn(2.f, odd), a, ib);
    *reinterpret_cast<float2*>(&hs[2 * q]) = h;
  }
  __syncthreads();

  // replicate padding of the high-rate signal at the two row ends
  const int64_t u_first = 2 * t0 - 6;  // u of hs[0]
  const int64_t u_last_needed = 2 * (t0 + kFirTile) + 5;
  if (u_first < 0 || u_last_needed >= 2 * T) {
    float left = 0.f, right = 0.f;
    if (u_first < 0) left = hs[-u_first];                      // u = 0
    if (u_last_needed >= 2 * T && 2 * T - 1 - u_first >= 0) right = hs[2 * T - 1 - u_first];
    __syncthreads();
    if (u_first < 0 && tid < 6) hs[tid] = left;                // u in [-6, -1]
    if (u_last_needed >= 2 * T && tid < 6) {
      const int64_t i = 2 * T - u_first + tid;                 // u in [2T, 2T+5]
      if (i >= 0 && i < 2 * kFirTile + 12) hs[i] = right;
    }
    __syncthreads();
  }

  // 3. low-pass, two outputs per thread
  float dn[12];
#pragma unroll
  for (int k = 0; k < 12; ++k) dn[k] = s_down[k];
  const int64_t valid = T - t0 < kFirTile ? T - t0 : kFirTile;
  for (int q = tid; 2 * q < valid; q += kFirThreads) {
    float w[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(&hs[4 * q + 4 * j]);
      w[4 * j] = v.x; w[4 * j + 1] = v.y; w[4 * j + 2] = v.z; w[4 * j + 3] = v.w;
    }
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int k = 0; k < 12; ++k) {
      y0 = fmaf(dn[k], w[k + 1], y0);
      y1 = fmaf(dn[k], w[k + 3], y1);
    }
    const int64_t t = t0 + 2 * q;
    const bool both = 2 * q + 1 < valid;
    if constexpr (kInt8Out) {
      const float sm = __ldg(p.smooth + c);
      int8_t* yrow = static_cast<int8_t*>(p.y) + row * T;
      yrow[t] = int8_rne_sat(__fdiv_rn(__fdiv_rn(y0, sm), p.scale));
      if (both) yrow[t + 1] = int8_rne_sat(__fdiv_rn(__fdiv_rn(y1, sm), p.scale));
    } else {
      float* yrow = static_cast<float*>(p.y) + row * T;
      if (both && ((row * T + t) & 1) == 0) {
        *reinterpret_cast<float2*>(yrow + t) = make_float2(y0, y1);
      } else {
        yrow[t] = y0;
        if (both) yrow[t + 1] = y1;
      }
    }
  }
}

}  // namespace isp
