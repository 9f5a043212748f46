// Fused row normalization -> quantization (memory-bound; kLanes = 16 or 32 lanes
// per row, i.e. two rows or one row per warp).
//
// Each lane owns groups of 8 consecutive elements (group g = sublane + kLanes i),
// so a row's lanes stream 8 kLanes contiguous elements per step with 16-byte loads
// (BF16) or two 16-byte loads (FP32).  Half-warp rows (K <= 512) give every lane
// twice the elements over which to spread the per-row reduction and scalar math.  The row statistic is accumulated in double from
// FP32 squares and rounded once; every following step is one IEEE FP32
// operation in the order of the reference module (see isp_b200.h for the
// reference file:line of each mode).
#pragma once

#include "common.cuh"

namespace isp {

struct NormQuantParams {
  const void* x;
  int64_t M;
  int K;
  const float* gamma;
  const float* bias;
  float eps;
  float out_mul;
  float scale;          // static scale (E4M3 / INT8) or NVFP4 global scale
  const float* smooth;  // INT8 SmoothQuant divisor or nullptr
  void* codes;
  void* scales_out;
  // AdaLN (RMS_GPTFAST only): y = ada_w[g] * norm(x) + ada_b[g], g = row / rows_per_group
  const float* ada_w;
  const float* ada_b;
  int64_t rows_per_group;
};

ISP_D void load_param8(const float* base, int g, float (&w)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(base + g * 8));
  const float4 b = __ldg(reinterpret_cast<const float4*>(base + g * 8 + 4));
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}

template <bool kBF16>
ISP_D void load_group(const void* row, int g, float (&v)[8]) {
  if constexpr (kBF16) {
    uint4 raw = ldg_nc_v4(static_cast<const uint16_t*>(row) + g * 8);
    bf16x8_to_f32(raw, v);
  } else {
    const float* p = static_cast<const float*>(row) + g * 8;
    uint4 a = ldg_nc_v4(p), b = ldg_nc_v4(p + 4);
    v[0] = __uint_as_float(a.x); v[1] = __uint_as_float(a.y);
    v[2] = __uint_as_float(a.z); v[3] = __uint_as_float(a.w);
    v[4] = __uint_as_float(b.x); v[5] = __uint_as_float(b.y);
    v[6] = __uint_as_float(b.z); v[7] = __uint_as_float(b.w);
  }
}

// Reductions over the kLanes lanes of a row (xor offsets stay inside the row).
template <int kLanes>
ISP_D double row_sum(double v) {
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <int kLanes>
ISP_D float row_max(float v) {
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One row's input as loaded (BF16: one 16-byte word per 8-element group; FP32: two),
// kept raw so the next row's loads can be in flight while this row is computed.
template <bool kBF16>
struct RawGroup {
  uint4 w[kBF16 ? 1 : 2];
};

template <bool kBF16, int kGroups, int kLanes>
ISP_D void load_row_raw(const NormQuantParams& p, int64_t row, int lane, RawGroup<kBF16> (&raw)[kGroups]) {
  if (row >= p.M) return;
  const int ngroups = p.K >> 3;
#pragma unroll
  for (int i = 0; i < kGroups; ++i) {
    const int g = lane + kLanes * i;
    if (g < ngroups) {
      if constexpr (kBF16) {
        raw[i].w[0] = ldg_nc_v4(static_cast<const uint16_t*>(p.x) + row * p.K + g * 8);
      } else {
        const float* q = static_cast<const float*>(p.x) + row * p.K + g * 8;
        raw[i].w[0] = ldg_nc_v4(q);
        raw[i].w[1] = ldg_nc_v4(q + 4);
      }
    }
  }
}

template <bool kBF16>
ISP_D void unpack_group(const RawGroup<kBF16>& r, float (&v)[8]) {
  if constexpr (kBF16) {
    bf16x8_to_f32(r.w[0], v);
  } else {
    v[0] = __uint_as_float(r.w[0].x); v[1] = __uint_as_float(r.w[0].y);
    v[2] = __uint_as_float(r.w[0].z); v[3] = __uint_as_float(r.w[0].w);
    v[4] = __uint_as_float(r.w[1].x); v[5] = __uint_as_float(r.w[1].y);
    v[6] = __uint_as_float(r.w[1].z); v[7] = __uint_as_float(r.w[1].w);
  }
}

// Normalization and quantization of one row whose values are in v (kLanes lanes;
// rows past M keep their lanes in the shuffles and skip every load and store).
template <bool kBF16, int kNorm, int kFmt, int kGroups, int kLanes>
ISP_D void norm_quant_row(const NormQuantParams& p, int64_t row, int lane, float (&v)[kGroups][8]) {
  const bool active = row < p.M;
  const int K = p.K;
  const int ngroups = active ? K >> 3 : 0;   // an inactive row owns no groups

  // ---- normalization ------------------------------------------------------
  if constexpr (kNorm != ISP_NORM_NONE) {
    // four independent double accumulators (no serial add chain); the FP32 squares
    // are summed exactly in double whatever the order, then rounded once
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
      const int g = lane + kLanes * i;
      if (g < ngroups) {
        float b8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if constexpr (kNorm == ISP_NORM_BIAS) load_param8(p.bias, g, b8);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float d = v[i][j];
          if constexpr (kNorm == ISP_NORM_BIAS) d = __fsub_rn(d, b8[j]);
          if constexpr (kBF16 && kNorm != ISP_NORM_BIAS) {
            // a BF16 value's square is exact in FP32 and in double: one double FMA
            acc[j & 3] = __fma_rn(static_cast<double>(d), static_cast<double>(d), acc[j & 3]);
          } else {
            acc[j & 3] += static_cast<double>(__fmul_rn(d, d));
          }
        }
      }
    }
    double ss = row_sum<kLanes>((acc[0] + acc[1]) + (acc[2] + acc[3]));
    const float mean = __fdiv_rn(static_cast<float>(ss), static_cast<float>(K));
    float r;
    if constexpr (kNorm == ISP_NORM_BIAS) {
      r = __fmul_rn(__fdiv_rn(1.f, __fsqrt_rn(mean)), p.out_mul);
    } else {
      r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(mean, p.eps)));
    }
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
      const int g = lane + kLanes * i;
      if (g < ngroups) {
        float gm[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
        if constexpr (kNorm == ISP_NORM_RMS_GPTFAST || kNorm == ISP_NORM_RMS_QWEN) load_param8(p.gamma, g, gm);
        float aw[8], ab[8];
        if (kNorm == ISP_NORM_RMS_GPTFAST && p.ada_w != nullptr) {
          const int64_t grp = row / p.rows_per_group;
          load_param8(p.ada_w + grp * K, g, aw);
          load_param8(p.ada_b + grp * K, g, ab);
        }
        if constexpr (kNorm == ISP_NORM_RMS_GPTFAST && kBF16) {
          // x * r and the product with gamma two elements per instruction (f32x2, each
          // lane rounded as the scalar op), the BF16 rounding of the pair in one conversion
          const float2 r2 = make_float2(r, r);
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float2 t = __fmul2_rn(make_float2(v[i][j], v[i][j + 1]), r2);
            const uint32_t h = pack_bf16_rn(t.x, t.y);
            float2 y = __fmul2_rn(make_float2(__uint_as_float(h << 16), __uint_as_float(h & 0xFFFF0000u)),
                                  make_float2(gm[j], gm[j + 1]));
            if (p.ada_w != nullptr) {   // scalar: a packed multiply-add may be contracted to one rounding
              y.x = __fadd_rn(__fmul_rn(aw[j], y.x), ab[j]);
              y.y = __fadd_rn(__fmul_rn(aw[j + 1], y.y), ab[j + 1]);
            }
            v[i][j] = y.x;
            v[i][j + 1] = y.y;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float y = __fmul_rn(v[i][j], r);
            if constexpr (kNorm == ISP_NORM_RMS_GPTFAST) {    // FP32 input: no intermediate rounding
              y = __fmul_rn(y, gm[j]);
              if (p.ada_w != nullptr) y = __fadd_rn(__fmul_rn(aw[j], y), ab[j]);
            } else if constexpr (kNorm == ISP_NORM_RMS_QWEN) {
              y = __fmul_rn(y, gm[j]);
              if constexpr (kBF16) y = bf16_round(y);
            } else {
              if constexpr (kBF16) y = bf16_round(y);
            }
            v[i][j] = y;
          }
        }
      }
    }
  }

  // ---- quantization -------------------------------------------------------
  if constexpr (kFmt == ISP_Q_E4M3_STATIC || kFmt == ISP_Q_E4M3_ROW) {
    float s = p.scale;
    if constexpr (kFmt == ISP_Q_E4M3_ROW) {
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < kGroups; ++i)
        if (lane + kLanes * i < ngroups)
#pragma unroll
          for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
      amax = row_max<kLanes>(amax);
      s = fmaxf(__fdiv_rn(amax, 448.f), 1e-12f);
      if (lane == 0 && active) static_cast<float*>(p.scales_out)[row] = s;
    }
    uint8_t* out = static_cast<uint8_t*>(p.codes) + row * K;
    const float rs = __frcp_rn(s);
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
      const int g = lane + kLanes * i;
      if (g < ngroups) {
        uint32_t w[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float* q = &v[i][4 * h];
          // satfinite == the reference's clamp(-448, 448) before the cast (NaN stays NaN)
          const float2 a = div_rn_recip2(make_float2(q[0], q[1]), s, rs);
          const float2 b = div_rn_recip2(make_float2(q[2], q[3]), s, rs);
          w[h] = static_cast<uint32_t>(e4m3x2(a.x, a.y)) | (static_cast<uint32_t>(e4m3x2(b.x, b.y)) << 16);
        }
        *reinterpret_cast<uint2*>(out + g * 8) = make_uint2(w[0], w[1]);
      }
    }
  } else if constexpr (kFmt == ISP_Q_INT8_STATIC) {
    int8_t* out = static_cast<int8_t*>(p.codes) + row * K;
    const float rscale = __frcp_rn(p.scale);
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
      const int g = lane + kLanes * i;
      if (g < ngroups) {
        uint32_t w[2] = {0u, 0u};
        float sm[8];
        if (p.smooth != nullptr) load_param8(p.smooth, g, sm);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float y = v[i][j];
          if (p.smooth != nullptr) y = __fdiv_rn(y, sm[j]);
          const int8_t q = int8_rne_sat(div_rn_recip(y, p.scale, rscale));
          w[j >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(q)) << (8 * (j & 3));
        }
        *reinterpret_cast<uint2*>(out + g * 8) = make_uint2(w[0], w[1]);
      }
    }
  } else {  // NVFP4: lanes (2p, 2p+1) hold the two halves of one 16-element block
    uint8_t* out = static_cast<uint8_t*>(p.codes) + row * (K / 2);
    // Row-major [M, K/16] scales, or the tensor-core layout (128-row x 4-block
    // chunks of 512 bytes, K chunks first): block b of row m sits at
    // ((m/128)*(K/64) + b/4)*512 + (m%32)*16 + ((m%128)/32)*4 + b%4.
    uint8_t* sf = kFmt == ISP_Q_NVFP4
                      ? static_cast<uint8_t*>(p.scales_out) + row * (K / 16)
                      : static_cast<uint8_t*>(p.scales_out) + (row >> 7) * (K / 64) * 512 + (row & 31) * 16 +
                            ((row >> 5) & 3) * 4;
    const float gscale = p.scale;
    const float six_g = __fmul_rn(6.f, gscale);
#pragma unroll
    for (int i = 0; i < kGroups; ++i) {
      const int g = lane + kLanes * i;
      // Every lane runs the shuffle; lanes without a group contribute 0.
      float amax = 0.f;
      if (g < ngroups)
#pragma unroll
        for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(v[i][j]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      if (g < ngroups) {
        float sb = __fdiv_rn(amax, six_g);
        if (sb == 0.f) sb = 1.f;
        const uint16_t sc2 = e4m3x2(fminf(sb, 448.f), 0.f);
        const uint8_t sc = static_cast<uint8_t>(sc2 & 0xFF);
        const float denom = __fmul_rn(e4m3_to_f32(sc), gscale);
        const float rden = __frcp_rn(denom);
        uint32_t packed = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) packed |= e2m1_code(div_rn_recip(v[i][j], denom, rden)) << (4 * j);
        *reinterpret_cast<uint32_t*>(out + g * 4) = packed;
        if ((g & 1) == 0) {
          const int b = g >> 1;
          if constexpr (kFmt == ISP_Q_NVFP4) sf[b] = sc;
          else sf[(b >> 2) * 512 + (b & 3)] = sc;
        }
      }
    }
  }
}

// kGroups: max 8-element groups per lane kept in registers (K <= 8 * kLanes * kGroups).
// Persistent blocks of 8 warps walk rows with a stride of the whole grid; each row's
// lanes issue the loads of their next row before normalizing and quantizing the current
// one, so HBM reads stay in flight while the row is computed.
template <bool kBF16, int kNorm, int kFmt, int kGroups, int kLanes>
__global__ void __launch_bounds__(256) norm_quant_kernel(NormQuantParams p) {
  static_assert(kLanes == 16 || kLanes == 32, "a row spans a half or a whole warp");
  const int lane = threadIdx.x % kLanes;   // lane within the row
  constexpr int kRowsPerBlock = 8 * (32 / kLanes);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kRowsPerBlock;
  int64_t row = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * (32 / kLanes) +
                (threadIdx.x & 31) / kLanes;
  pdl_wait();       // predecessor's output (this kernel's input) complete and visible
  pdl_trigger();
  if (__all_sync(0xffffffffu, row >= p.M)) return;
  RawGroup<kBF16> raw[kGroups];
  load_row_raw<kBF16, kGroups, kLanes>(p, row, lane, raw);
  for (;;) {
    float v[kGroups][8];
#pragma unroll
    for (int i = 0; i < kGroups; ++i) unpack_group<kBF16>(raw[i], v[i]);
    const int64_t next = row + stride;
    load_row_raw<kBF16, kGroups, kLanes>(p, next, lane, raw);   // in flight during this row
    norm_quant_row<kBF16, kNorm, kFmt, kGroups, kLanes>(p, row, lane, v);
    row = next;
    if (__all_sync(0xffffffffu, row >= p.M)) break;
  }
}

// Persistent grid: as many blocks as are resident at once (at most one per 16 or 8 rows).
template <typename Kern>
int launch_norm_quant_persistent(Kern kern, int64_t rows_per_block, const NormQuantParams& p, cudaStream_t stream) {
  static int per_sm[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int occ = dev >= 0 && dev < 64 ? per_sm[dev] : 0;
  if (occ == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, 256, 0) != cudaSuccess || occ < 1) {
      cudaGetLastError();
      occ = 1;
    }
    if (dev >= 0 && dev < 64) per_sm[dev] = occ;
  }
  const int64_t need = (p.M + rows_per_block - 1) / rows_per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * occ;
  return launch_pdl(kern, dim3(static_cast<unsigned>(need < cap ? need : cap)), dim3(256), 0, stream, p);
}

template <bool kBF16, int kNorm, int kFmt>
int launch_norm_quant_groups(const NormQuantParams& p, cudaStream_t stream) {
  if (p.K <= 512) {   // half-warp rows: 16 rows per block, up to 4 groups per lane
    if (p.K <= 256) return launch_norm_quant_persistent(norm_quant_kernel<kBF16, kNorm, kFmt, 2, 16>, 16, p, stream);
    return launch_norm_quant_persistent(norm_quant_kernel<kBF16, kNorm, kFmt, 4, 16>, 16, p, stream);
  }
  const int per_lane = (p.K / 8 + 31) / 32;
  if (per_lane <= 4) return launch_norm_quant_persistent(norm_quant_kernel<kBF16, kNorm, kFmt, 4, 32>, 8, p, stream);
  if (per_lane <= 8) return launch_norm_quant_persistent(norm_quant_kernel<kBF16, kNorm, kFmt, 8, 32>, 8, p, stream);
  if (per_lane <= 16) return launch_norm_quant_persistent(norm_quant_kernel<kBF16, kNorm, kFmt, 16, 32>, 8, p, stream);
  if constexpr (kNorm == ISP_NORM_NONE) {
    if (per_lane <= 32)
      return launch_norm_quant_persistent(norm_quant_kernel<kBF16, kNorm, kFmt, 32, 32>, 8, p, stream);
  }
  return ISP_ERR_SHAPE;
}

template <bool kBF16, int kNorm>
int launch_norm_quant_fmt(int fmt, const NormQuantParams& p, cudaStream_t s) {
  switch (fmt) {
    case ISP_Q_E4M3_STATIC: return launch_norm_quant_groups<kBF16, kNorm, ISP_Q_E4M3_STATIC>(p, s);
    case ISP_Q_E4M3_ROW: return launch_norm_quant_groups<kBF16, kNorm, ISP_Q_E4M3_ROW>(p, s);
    case ISP_Q_INT8_STATIC: return launch_norm_quant_groups<kBF16, kNorm, ISP_Q_INT8_STATIC>(p, s);
    case ISP_Q_NVFP4: return launch_norm_quant_groups<kBF16, kNorm, ISP_Q_NVFP4>(p, s);
    case ISP_Q_NVFP4_MMA: return launch_norm_quant_groups<kBF16, kNorm, ISP_Q_NVFP4_MMA>(p, s);
    default: return ISP_ERR_ARG;
  }
}

template <bool kBF16>
int launch_norm_quant_kind(int kind, int fmt, const NormQuantParams& p, cudaStream_t s) {
  switch (kind) {
    case ISP_NORM_NONE: return launch_norm_quant_fmt<kBF16, ISP_NORM_NONE>(fmt, p, s);
    case ISP_NORM_RMS_GPTFAST: return launch_norm_quant_fmt<kBF16, ISP_NORM_RMS_GPTFAST>(fmt, p, s);
    case ISP_NORM_RMS_QWEN: return launch_norm_quant_fmt<kBF16, ISP_NORM_RMS_QWEN>(fmt, p, s);
    case ISP_NORM_BIAS: return launch_norm_quant_fmt<kBF16, ISP_NORM_BIAS>(fmt, p, s);
    default: return ISP_ERR_ARG;
  }
}

}  // namespace isp
