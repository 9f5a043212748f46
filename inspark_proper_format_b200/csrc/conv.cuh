// Quantized learned Conv1d / ConvTranspose1d: the kernels around the implicit
// GEMM (which is gemm_kernel with EPI_CONV).
//
//   conv_amax_kernel   per-utterance max |x| (dynamic input scale of the FP8 path)
//   conv_quant_kernel  x [B, C, T] (FP32 or BF16, channels first, the vocoder's
//                      layout) -> channels-last codes [B, T_rows, C_pad] with the
//                      static or per-utterance scale; rows >= T and channels >= C
//                      coded 0.  Channels-last makes every (tap, 128-channel) slice
//                      of the A operand one TMA box at a shifted row, so the GEMM
//                      gathers the convolution windows with tiled loads and rows
//                      outside the utterance read as zero (the zero padding).
//   conv_pack_kernel   per-output-channel weight codes [CI * KW, ldw] (the packed
//                      [K, N] layout of quantization/weights.py:5-17) -> the
//                      phase-folded B operand [CO * phases, taps, C_pad].
#pragma once

#include "common.cuh"
#include "gemm_sm100.cuh"

namespace isp {

// ---- per-utterance amax ------------------------------------------------------
// grid (blocks_per_utterance, B); amax[b] must start at +0 (the host clears it).
// Non-negative floats order like their bit patterns, so an unsigned atomicMax
// on the bits is the float maximum.
template <bool kBf16>
__global__ void __launch_bounds__(256) conv_amax_kernel(const void* x, int64_t per_utt, float* amax) {
  const int64_t base = static_cast<int64_t>(blockIdx.y) * per_utt;
  float m = 0.f;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per_utt;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v;
    if constexpr (kBf16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[base + i]);
    else v = __ldg(static_cast<const float*>(x) + base + i);
    m = fmaxf(m, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    atomicMax(reinterpret_cast<unsigned int*>(amax) + blockIdx.y, __float_as_uint(m));
  }
}

// ---- quantize + transpose to channels-last -----------------------------------
struct ConvQuantParams {
  const void* x;           // [B, C, T]
  int64_t B;
  int C;
  int64_t T;
  int64_t t_rows;          // rows written per utterance (>= T; rows >= T are zero)
  int c_pad;
  int chunks;              // c_pad / 16
  float scale;             // static input scale (amax == nullptr)
  float rscale;            // RN(1 / scale)
  const float* amax;       // dynamic: per-utterance max |x|, scale = max(amax / 448, 1e-12)
  const float* smooth;     // INT8: per-channel SmoothQuant divisor, or nullptr
  uint8_t* xq;             // [B, t_rows, c_pad]
};

// One thread per (row, 16 channels); lanes take consecutive rows, so every
// per-channel read of x is one contiguous row segment.
template <bool kInt8, bool kBf16>
__global__ void __launch_bounds__(256) conv_quant_kernel(ConvQuantParams p) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = p.B * p.chunks * p.t_rows;
  if (i >= total) return;
  const int64_t t = i % p.t_rows;
  const int64_t rest = i / p.t_rows;
  const int chunk = static_cast<int>(rest % p.chunks);
  const int64_t b = rest / p.chunks;
  float scale = p.scale, rscale = p.rscale;
  if (p.amax != nullptr) {
    scale = gemm::conv_dynamic_scale(__ldg(p.amax + b));
    rscale = __frcp_rn(scale);
  }
  uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int c = chunk * 16 + j;
    float v = 0.f;
    if (t < p.T && c < p.C) {
      const int64_t off = (b * p.C + c) * p.T + t;
      if constexpr (kBf16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(p.x)[off]);
      else v = __ldg(static_cast<const float*>(p.x) + off);
    }
    uint32_t code;
    if constexpr (kInt8) {
      if (p.smooth != nullptr && c < p.C) v = __fdiv_rn(v, __ldg(p.smooth + c));
      code = static_cast<uint8_t>(int8_rne_sat(div_rn_recip(v, scale, rscale)));
    } else {
      // satfinite == the reference's clamp(-448, 448) before the cast
      code = e4m3x2(div_rn_recip(v, scale, rscale), 0.f) & 0xFFu;
    }
    w[j >> 2] |= code << (8 * (j & 3));
  }
  *reinterpret_cast<uint4*>(p.xq + (b * p.t_rows + t) * p.c_pad + chunk * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

// ---- weight packing ----------------------------------------------------------
// B operand of the phase-folded GEMM: row co * P + r, K = (window slot j, channel c).
// Conv1d (P = 1): slot j is tap j.  ConvTranspose1d (stride S = P): slot j reads input
// row q + (r_min + j) for output time q * S + r, which tap k = (r + padding - (r_min + j)
// * S) / dilation supplies when that division is exact and 0 <= k < KW; otherwise 0.
struct ConvPackParams {
  const uint8_t* src;      // [CI * KW, ldw] codes, row ci * KW + tap, column co
  int64_t ldw;
  int CO, CI, KW;
  int phases, taps, c_pad;
  int transposed, stride, dilation, padding, r_min;
  uint8_t* dst;            // [CO * phases, taps, c_pad]
};

// One thread per 16 destination bytes (16 channels of one (row, slot)).
__global__ void __launch_bounds__(256) conv_pack_kernel(ConvPackParams p) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int chunks = p.c_pad / 16;
  const int64_t total = static_cast<int64_t>(p.CO) * p.phases * p.taps * chunks;
  if (i >= total) return;
  const int chunk = static_cast<int>(i % chunks);
  int64_t rest = i / chunks;
  const int slot = static_cast<int>(rest % p.taps);
  const int64_t row = rest / p.taps;
  const int co = static_cast<int>(row / p.phases);
  const int r = static_cast<int>(row % p.phases);
  int tap = slot;
  if (p.transposed) {
    const int64_t num = static_cast<int64_t>(r) + p.padding - static_cast<int64_t>(p.r_min + slot) * p.stride;
    tap = (num >= 0 && num % p.dilation == 0 && num / p.dilation < p.KW) ? static_cast<int>(num / p.dilation) : -1;
  }
  uint32_t w[4] = {0u, 0u, 0u, 0u};
  if (tap >= 0) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int c = chunk * 16 + j;
      if (c < p.CI) w[j >> 2] |= static_cast<uint32_t>(p.src[(static_cast<int64_t>(c) * p.KW + tap) * p.ldw + co])
                                 << (8 * (j & 3));
    }
  }
  *reinterpret_cast<uint4*>(p.dst + i * 16) = make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace isp
