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
// on the bits is the float maximum.  fmaxf drops NaN operands, as the reference's
// tl.max does (Triton's default maxnum semantics, ops/triton/fp8_conv.py:10,15-16):
// NaN inputs leave the utterance's scale finite and propagate only through their
// own codes.
template <bool kBf16>
__global__ void __launch_bounds__(256) conv_amax_kernel(const void* x, int64_t per_utt, float* amax) {
  const int64_t base = static_cast<int64_t>(blockIdx.y) * per_utt;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  float m = 0.f;
  if constexpr (kBf16) {
    const __nv_bfloat16* xs = static_cast<const __nv_bfloat16*>(x) + base;
    // 16-byte loads (8 values) when the utterance starts 16-byte aligned
    if ((reinterpret_cast<uintptr_t>(xs) & 15) == 0) {
      const int64_t n8 = per_utt / 8;
      for (int64_t i = first; i < n8; i += stride) {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(xs) + i);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[j] << 16)),
                                                       fabsf(__uint_as_float(w[j] & 0xFFFF0000u))));
      }
      for (int64_t i = n8 * 8 + first; i < per_utt; i += stride) m = fmaxf(m, fabsf(__bfloat162float(xs[i])));
    } else {
      for (int64_t i = first; i < per_utt; i += stride) m = fmaxf(m, fabsf(__bfloat162float(xs[i])));
    }
  } else {
    const float* xs = static_cast<const float*>(x) + base;
    if ((reinterpret_cast<uintptr_t>(xs) & 15) == 0) {
      const int64_t n4 = per_utt / 4;
      for (int64_t i = first; i < n4; i += stride) {
        const float4 q = __ldg(reinterpret_cast<const float4*>(xs) + i);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(q.x), fabsf(q.y)), fmaxf(fabsf(q.z), fabsf(q.w))));
      }
      for (int64_t i = n4 * 4 + first; i < per_utt; i += stride) m = fmaxf(m, fabsf(__ldg(xs + i)));
    } else {
      for (int64_t i = first; i < per_utt; i += stride) m = fmaxf(m, fabsf(__ldg(xs + i)));
    }
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
  float scale;             // static input scale (amax == nullptr)
  float rscale;            // RN(1 / scale)
  const float* amax;       // dynamic: per-utterance max |x|, scale = max(amax / 448, 1e-12)
  const float* smooth;     // INT8: per-channel SmoothQuant divisor, or nullptr
  uint8_t* xq;             // [B, t_rows, c_pad]
};

// A block transposes one tile of 64 rows x 128 channels through shared memory:
// loads walk time (a warp reads 32 consecutive samples of one channel, 128 bytes),
// each thread codes 4 channels of one row into a word at [row][channel / 4] (row
// pitch 33 words: conflict-free), and stores walk channels (a warp writes one
// 128-byte channels-last row).  grid (ceil(t_rows / 64), c_pad / 128, B).
constexpr int kCqRows = 64;
constexpr int kCqPitch = 33;                 // words per staged row (32 + 1 pad)

template <bool kBf16>
ISP_D float conv_load(const void* x, int64_t off) {
  if constexpr (kBf16) return __bfloat162float(static_cast<const __nv_bfloat16*>(x)[off]);
  else return __ldg(static_cast<const float*>(x) + off);
}

template <bool kInt8, bool kBf16>
__global__ void __launch_bounds__(256) conv_quant_kernel(ConvQuantParams p) {
  __shared__ uint32_t tile[kCqRows * kCqPitch];
  const int64_t b = blockIdx.z;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kCqRows;
  const int c0 = blockIdx.y * 128;
  float scale = p.scale, rscale = p.rscale;
  if (p.amax != nullptr) {
    scale = gemm::conv_dynamic_scale(__ldg(p.amax + b));
    rscale = __frcp_rn(scale);
  }
  // thread -> row r (fixed) and channel groups quad0 + 4i; the block's first element
  const int r = threadIdx.x % kCqRows;
  const int quad0 = threadIdx.x / kCqRows;
  const int64_t t = t0 + r;
  const int64_t base = (b * p.C + c0) * p.T + t;
  const bool interior = t0 + kCqRows <= p.T && c0 + 128 <= p.C;   // block-uniform
  // FP32 interior tiles with 16-byte aligned rows: a thread takes 4 consecutive rows x 4
  // channels and reads each channel's 4 samples as one float4 (half-warps cover 256
  // contiguous bytes of one channel); block-uniform.
  if constexpr (!kBf16) {
    if (interior && (p.T & 3) == 0 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int k = threadIdx.x + 256 * i;
        const int rg = k % (kCqRows / 4);          // group of 4 rows
        const int quad = k / (kCqRows / 4);        // group of 4 channels
        const float* src = static_cast<const float*>(p.x) + (b * p.C + c0 + quad * 4) * p.T + t0 + 4 * rg;
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __ldg(reinterpret_cast<const float4*>(src + j * p.T));
        float col[4][4];   // [row][channel]
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          col[0][j] = v[j].x;
          col[1][j] = v[j].y;
          col[2][j] = v[j].z;
          col[3][j] = v[j].w;
        }
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          uint32_t word;
          if constexpr (kInt8) {
            word = 0u;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float u = col[rr][j];
              if (p.smooth != nullptr) u = __fdiv_rn(u, __ldg(p.smooth + c0 + quad * 4 + j));
              word |= static_cast<uint32_t>(static_cast<uint8_t>(int8_rne_sat(div_rn_recip(u, scale, rscale))))
                      << (8 * j);
            }
          } else {
            word = static_cast<uint32_t>(e4m3x2(div_rn_recip(col[rr][0], scale, rscale),
                                                div_rn_recip(col[rr][1], scale, rscale))) |
                   static_cast<uint32_t>(e4m3x2(div_rn_recip(col[rr][2], scale, rscale),
                                                div_rn_recip(col[rr][3], scale, rscale)))
                       << 16;
          }
          tile[(4 * rg + rr) * kCqPitch + quad] = word;
        }
      }
      __syncthreads();
#pragma unroll 2
      for (int k = threadIdx.x; k < kCqRows * 32; k += 256) {
        const int rr = k / 32;
        const int w = k % 32;
        reinterpret_cast<uint32_t*>(p.xq + (b * p.t_rows + t0 + rr) * p.c_pad + c0)[w] = tile[rr * kCqPitch + w];
      }
      return;
    }
  }
#pragma unroll 2
  for (int i = 0; i < 8; ++i) {
    const int quad = quad0 + 4 * i;
    const int64_t off = base + static_cast<int64_t>(quad * 4) * p.T;
    float v[4];
    if (interior) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = conv_load<kBf16>(p.x, off + j * p.T);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = (t < p.T && c0 + quad * 4 + j < p.C) ? conv_load<kBf16>(p.x, off + j * p.T) : 0.f;
    }
    uint32_t word;
    if constexpr (kInt8) {
      word = 0u;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = c0 + quad * 4 + j;
        float u = v[j];
        if (p.smooth != nullptr && c < p.C) u = __fdiv_rn(u, __ldg(p.smooth + c));
        word |= static_cast<uint32_t>(static_cast<uint8_t>(int8_rne_sat(div_rn_recip(u, scale, rscale)))) << (8 * j);
      }
    } else {
      // satfinite == the reference's clamp(-448, 448) before the cast
      word = static_cast<uint32_t>(e4m3x2(div_rn_recip(v[0], scale, rscale), div_rn_recip(v[1], scale, rscale))) |
             static_cast<uint32_t>(e4m3x2(div_rn_recip(v[2], scale, rscale), div_rn_recip(v[3], scale, rscale)))
                 << 16;
    }
    tile[r * kCqPitch + quad] = word;
  }
  __syncthreads();
#pragma unroll 2
  for (int k = threadIdx.x; k < kCqRows * 32; k += 256) {
    const int rr = k / 32;
    const int w = k % 32;
    const int64_t tt = t0 + rr;
    if (tt < p.t_rows)
      reinterpret_cast<uint32_t*>(p.xq + (b * p.t_rows + tt) * p.c_pad + c0)[w] = tile[rr * kCqPitch + w];
  }
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
