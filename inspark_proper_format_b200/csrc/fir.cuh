// BigVGAN anti-aliased Snake activation, fused: 2x polyphase upsample ->
// Snake -> stride-2 low-pass, one pass over x, FP32 throughout.
//
// A tile is kFirTile consecutive outputs of one row (row = b*C + c):
//   1. xs[j] = x[clamp(t0 - 8 + j, 0, T-1)]  (replicate padding by clamping).
//   2. hs[i] = Snake(U[u]) for u = 2 t0 - 6 + i, computed per (even u, odd u)
//      pair q (u = 2s, 2s+1 with s = t0 - 3 + q) from xs[q+2 .. q+8]:
//        U[2s]   = 2 sum_j up[2j+1] x[s+2-j],   U[2s+1] = 2 sum_j up[2j] x[s+3-j].
//      Entries with u outside [0, 2T) then take the value at the clamped
//      index (the replicate padding in front of the low-pass).
//   3. y[t0+o] = sum_k down[k] hs[2o + k + 1].
// This is the index algebra of ops/triton/vocoder_tiled_fir.py:20-39 and
// ops/triton/alias_free.py:7-26, evaluated once per high-rate sample.
//
// The 24 filter taps travel by value in the kernel parameters, so every FMA
// reads its coefficient from the constant bank: no registers are spent on
// them.  The kernel is persistent; while tile i computes, the low-rate halo
// of tile i+1 streams in by a 1-D bulk async copy (row length T % 4 == 0).
#pragma once

#include "common.cuh"

namespace isp {

#ifndef ISP_FIR_TILE
#define ISP_FIR_TILE 1024
#endif
#ifndef ISP_FIR_THREADS
#define ISP_FIR_THREADS 86
#endif
#ifndef ISP_FIR_MIN_BLOCKS
#define ISP_FIR_MIN_BLOCKS 12
#endif
#ifndef ISP_FIR_MUFU_SIN
#define ISP_FIR_MUFU_SIN 1
#endif
// Outputs per tile (a power of two divides the vocoder's row lengths evenly).
// The tile's 1030 high-rate pairs form 258 quads: 86 threads take exactly three
// each, so no thread idles at the phase barrier.  Small blocks (16.6 KB of shared
// memory, 12-13 resident per SM) let one block's phase barrier overlap the others'
// work: measured 1.51 ms per B64 micro-batch against 1.69 ms with 4096-output
// tiles of 342 threads (3 per SM), same results.
constexpr int kFirTile = ISP_FIR_TILE;
constexpr int kFirThreads = ISP_FIR_THREADS;
constexpr int kFirQuads = (kFirTile + 6 + 3) / 4;      // quads of high-rate pairs per full tile
constexpr int kFirXs = 4 * kFirQuads + 8;              // low-rate halo buffer (floats): reads reach 4 quads + 7
constexpr int kFirHs = 8 * kFirQuads;                  // high-rate buffer (floats): 8 samples per quad
static_assert(kFirXs >= kFirTile + 16 && kFirTile % 4 == 0, "FIR tile geometry");
constexpr int kFirSmemBytes = (2 * kFirXs + kFirHs) * 4;

struct FirParams {
  const float* x;
  int64_t rows;
  int C;
  int64_t T;
  int64_t tiles_per_row;
  const float* alpha;
  const float* inv_beta;
  void* y;
  const float* smooth;
  float scale;
  float rscale;    // RN(1 / scale)
  // Persistent walk over tiles without division: with G = gridDim.x blocks,
  // one step advances the tile index by G, i.e. the row by g_rows (and one
  // more on carry), the tile-in-row by g_tiles and the channel by g_chan.
  int g_rows, g_tiles, g_chan;
  float up2[12];   // 2 * up: the upsampler's gain of 2 folded in (exact)
  float down[12];
  // Packed copies for the f32x2 FMAs: upp[m] = (up2[11 - 2m], up2[10 - 2m]) pairs the
  // even and odd polyphase sums; dnp[i] = (down[2i + 1], down[2i + 2]) pairs adjacent taps.
  float2 upp[6];
  float2 dnp[5];
};

// Position of a tile: row (= b*C + c), tile index within the row, channel.
struct FirPos {
  int64_t row;
  int tr;
  int c;
  ISP_D void advance(const FirParams& p) {
    tr += p.g_tiles;
    row += p.g_rows;
    c += p.g_chan;
    if (tr >= p.tiles_per_row) {
      tr -= static_cast<int>(p.tiles_per_row);
      row += 1;
      c += 1;
    }
    if (c >= p.C) c -= p.C;
  }
};

// sin(x)^2, valid for |x| <= kSinFastLimit.
// Method: Cody-Waite reduction modulo pi (sin^2 has period pi) with a two-term
// split of pi, r = x - k pi in [-pi/2, pi/2], then sin(r) = r + r^3 P(r^2)
// with a degree-4 P fitted for this library (minimax relative error on
// [0, pi/2] by Lawson's iteratively reweighted least squares); about 2 ulp on
// the reduced range.  k = rint(x / pi) uses the 1.5 * 2^23 rounding constant,
// exact while |x / pi| < 2^22.  Wider arguments are handled by the caller
// with CUDA's sinf (see the tile fallback in fir_snake_kernel).
constexpr float kSinFastLimit = 1.0e6f;

ISP_D float sin_squared(float x) {
  constexpr float kInvPi = 0x1.45f306p-2f;
  constexpr float kPiHi = 0x1.921fb6p+1f;       // float(pi)
  constexpr float kPiLo = -0x1.777a5cp-24f;     // pi - float(pi)
  constexpr float kRound = 12582912.0f;         // 1.5 * 2^23
  const float k = fmaf(x, kInvPi, kRound) - kRound;
  float r = fmaf(k, -kPiHi, x);
  r = fmaf(k, -kPiLo, r);
#if ISP_FIR_MUFU_SIN
  // CUDA's __sinf on the reduced argument |r| <= pi/2 (documented maximum
  // absolute error 2^-21.41 on [-pi, pi]); it runs on the MUFU pipe and
  // leaves the FMA pipe to the filters.
  const float s = __sinf(r);
  return s * s;
#else
  const float r2 = r * r;
  float p = fmaf(-0x1.9a6886p-26f, r2, 0x1.71708p-19f);
  p = fmaf(p, r2, -0x1.a017dap-13f);
  p = fmaf(p, r2, 0x1.11110cp-7f);
  p = fmaf(p, r2, -0x1.555556p-3f);
  const float s = fmaf(r * r2, p, r);
  return s * s;
#endif
}

// Snake v + inv_beta * sin(alpha v)^2 (the product then the sum, fused);
// `wide` collects max |alpha v| so the caller can detect the rare argument
// beyond the polynomial's range.
ISP_D float snake(float v, float a, float ib, float& wide) {
  const float t = v * a;
  wide = fmaxf(wide, fabsf(t));
  return fmaf(ib, sin_squared(t), v);
}
ISP_D float snake_wide(float v, float a, float ib) {
  const float s = sinf(v * a);
  return fmaf(ib, s * s, v);
}

ISP_D uint32_t fir_smem_u32(const void* ptr) { return static_cast<uint32_t>(__cvta_generic_to_shared(ptr)); }

// Bounded wait on an mbarrier phase (true on success).
ISP_D bool fir_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(ok)
      : "r"(fir_smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
ISP_D bool fir_wait(uint64_t* bar, uint32_t parity) {
  if (fir_try(bar, parity)) return true;
  const uint64_t start = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (fir_try(bar, parity)) return true;
    if ((i & 63u) == 63u && globaltimer() - start > kWaitLimitNs) return false;
  }
}

// x[row, lo .. hi) -> xs buffer, asynchronously (1-D bulk copy, 16-byte granules).
// xs[i] holds x[clamp(t0 - 8 + i)]; the in-range part [lo, hi) arrives here and
// the clamped ends are filled after the copy lands.
ISP_D void fir_issue_tile(const FirParams& p, const FirPos& pos, float* xs, uint64_t* bar) {
  const int64_t row = pos.row;
  const int64_t t0 = static_cast<int64_t>(pos.tr) * kFirTile;
  const int64_t lo = t0 - 8 < 0 ? 0 : t0 - 8;
  const int64_t hi = t0 + kFirTile + 8 > p.T ? p.T : t0 + kFirTile + 8;
  const uint32_t bytes = static_cast<uint32_t>((hi - lo) * 4);
  float* dst = xs + (lo - (t0 - 8));
  const float* src = p.x + row * p.T + lo;
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fir_smem_u32(bar)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   fir_smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(fir_smem_u32(bar))
               : "memory");
}

// Persistent: each block walks tiles blockIdx.x, +gridDim.x, ...  With kBulk
// (T % 4 == 0) the halo of tile i+1 streams into the other buffer while tile i
// computes; otherwise each tile's halo is read with clamped scalar loads.
template <bool kInt8Out, bool kBulk>
__global__ void __launch_bounds__(kFirThreads, ISP_FIR_MIN_BLOCKS)
    fir_snake_kernel(const __grid_constant__ FirParams p) {
  extern __shared__ __align__(16) float fir_smem[];
  float* const xs0 = fir_smem;
  float* const xs1 = fir_smem + kFirXs;
  float* const hs = fir_smem + 2 * kFirXs;
  __shared__ __align__(8) uint64_t bar[2];

  const int tid = threadIdx.x;
  const int64_t T = p.T;
  const int64_t total = p.rows * p.tiles_per_row;
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(fir_smem_u32(&bar[0])));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(fir_smem_u32(&bar[1])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  uint32_t phase0 = 0u, phase1 = 0u;
  bool pending0 = false, pending1 = false;
  int64_t tile = blockIdx.x;
  FirPos pos;                                    // one division per thread, at start
  pos.row = tile / p.tiles_per_row;
  pos.tr = static_cast<int>(tile - pos.row * p.tiles_per_row);
  pos.c = static_cast<int>(pos.row % p.C);
  if constexpr (kBulk) {
    if (tile < total && tid == 0) fir_issue_tile(p, pos, xs0, &bar[0]);
    pending0 = tile < total;
  }
  int buf = 0;
  for (; tile < total; tile += gridDim.x, buf ^= 1, pos.advance(p)) {
    const int64_t row = pos.row;
    const int64_t t0 = static_cast<int64_t>(pos.tr) * kFirTile;
    float* const xs = buf ? xs1 : xs0;
    if constexpr (kBulk) {
      const int64_t next = tile + gridDim.x;
      if (next < total) {
        FirPos np = pos;
        np.advance(p);
        if (tid == 0) fir_issue_tile(p, np, buf ? xs0 : xs1, &bar[buf ^ 1]);
        if (buf) pending0 = true;
        else pending1 = true;
      }
      const bool ok = fir_wait(&bar[buf], buf ? phase1 : phase0);
      if (__syncthreads_or(!ok)) {               // block-uniform: give up together
        if (tid == 0) record_timeout();
        break;
      }
      if (buf) {
        phase1 ^= 1u;
        pending1 = false;
      } else {
        phase0 ^= 1u;
        pending0 = false;
      }
    } else {
      const float* xrow = p.x + row * T;
      for (int j = tid; j < kFirXs; j += kFirThreads) {
        int64_t t = t0 - 8 + j;
        t = t < 0 ? 0 : (t >= T ? T - 1 : t);
        xs[j] = __ldg(xrow + t);
      }
      __syncthreads();
    }

    const int c = pos.c;
    const float a = __ldg(p.alpha + c);
    const float ib = __ldg(p.inv_beta + c);

    // clamped ends of the halo (replicate padding)
    if constexpr (kBulk) {
      const int64_t lo = t0 - 8 < 0 ? 0 : t0 - 8;
      const int64_t hi = t0 + kFirTile + 8 > T ? T : t0 + kFirTile + 8;
      const int first = static_cast<int>(lo - (t0 - 8));     // xs index of x[lo]
      const int last = static_cast<int>(hi - 1 - (t0 - 8));  // xs index of x[hi - 1]
      if (first > 0 || last < kFirXs - 1) {
        const float xl = xs[first], xr = xs[last];
        for (int i = tid; i < kFirXs; i += kFirThreads) {
          if (i < first) xs[i] = xl;
          else if (i > last) xs[i] = xr;
        }
        __syncthreads();
      }
    }

    // high-rate samples: each thread takes four consecutive pairs q0 .. q0+3
    // from the window w = xs[q0 .. q0+11]; pair q0+d reads w[d+2 .. d+8].
    const int valid = static_cast<int>(T - t0 < kFirTile ? T - t0 : kFirTile);
    const int quads = (valid + 6 + 3) / 4;
    float wide = 0.f;
    for (int qq = tid; qq < quads; qq += kFirThreads) {
      const int q0 = 4 * qq;
      float w[12];
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(&xs[q0 + 4 * j]);
        w[4 * j] = v.x;
        w[4 * j + 1] = v.y;
        w[4 * j + 2] = v.z;
        w[4 * j + 3] = v.w;
      }
      float h[8];
#pragma unroll
      for (int d = 0; d < 4; ++d) {
        // (even, odd) in one f32x2 accumulator: the same FMAs in the same order
        float2 eo = make_float2(0.f, 0.f);
#pragma unroll
        for (int m = 0; m < 6; ++m) eo = __ffma2_rn(p.upp[m], make_float2(w[d + 2 + m], w[d + 3 + m]), eo);
        h[2 * d] = snake(eo.x, a, ib, wide);
        h[2 * d + 1] = snake(eo.y, a, ib, wide);
      }
      *reinterpret_cast<float4*>(&hs[2 * q0]) = make_float4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<float4*>(&hs[2 * q0 + 4]) = make_float4(h[4], h[5], h[6], h[7]);
    }
    // Rare: some |alpha v| left the polynomial's range; redo this tile's
    // high-rate samples with CUDA's sinf (block-uniform decision).
    if (__syncthreads_or(!(wide <= kSinFastLimit))) {
      for (int q = tid; q < 4 * quads; q += kFirThreads) {
        float even = 0.f, odd = 0.f;
#pragma unroll
        for (int m = 0; m < 6; ++m) {
          even = fmaf(p.up2[11 - 2 * m], xs[q + 2 + m], even);
          odd = fmaf(p.up2[10 - 2 * m], xs[q + 3 + m], odd);
        }
        hs[2 * q] = snake_wide(even, a, ib);
        hs[2 * q + 1] = snake_wide(odd, a, ib);
      }
      __syncthreads();
    }

    // replicate padding of the high-rate signal at the two row ends
    const int64_t u_first = 2 * t0 - 6;  // u of hs[0]
    const int64_t u_last_needed = 2 * (t0 + kFirTile) + 5;
    if (u_first < 0 || u_last_needed >= 2 * T) {
      float left = 0.f, right = 0.f;
      if (u_first < 0) left = hs[-u_first];                    // u = 0
      if (u_last_needed >= 2 * T) right = hs[2 * T - 1 - u_first];
      __syncthreads();
      if (u_first < 0 && tid < 6) hs[tid] = left;              // u in [-6, -1]
      if (u_last_needed >= 2 * T && tid < 6) {
        const int64_t i = 2 * T - u_first + tid;               // u in [2T, 2T+5]
        if (i >= 0 && i < kFirHs) hs[i] = right;
      }
      __syncthreads();
    }

    // low-pass, four outputs per thread from w = hs[8q .. 8q+19]: y[4q + o] =
    // down[0] w[2o+1] + sum_i (down[2i+1], down[2i+2]) . (w[2o+2i+2], w[2o+2i+3]) +
    // down[11] w[2o+12], the tap pairs as f32x2 FMAs on aligned sample pairs
    float* const yrow_f = static_cast<float*>(p.y) + row * T + t0;
    int8_t* const yrow_i = static_cast<int8_t*>(p.y) + row * T + t0;
    float rsm = 1.f, sm = 1.f;
    if constexpr (kInt8Out) {
      sm = __ldg(p.smooth + c);
      rsm = __frcp_rn(sm);
    }
    for (int q = tid; 4 * q < valid; q += kFirThreads) {
      float w[20];
#pragma unroll
      for (int j = 0; j < 5; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(&hs[8 * q + 4 * j]);
        w[4 * j] = v.x;
        w[4 * j + 1] = v.y;
        w[4 * j + 2] = v.z;
        w[4 * j + 3] = v.w;
      }
      float y[4];
#pragma unroll
      for (int o = 0; o < 4; ++o) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 5; ++i) acc = __ffma2_rn(p.dnp[i], make_float2(w[2 * o + 2 * i + 2], w[2 * o + 2 * i + 3]), acc);
        y[o] = fmaf(p.down[11], w[2 * o + 12], fmaf(p.down[0], w[2 * o + 1], acc.x + acc.y));
      }
      const int t = 4 * q;
      const int n = valid - t < 4 ? valid - t : 4;
      if constexpr (kInt8Out) {
        int8_t qv[4];
#pragma unroll
        for (int o = 0; o < 4; ++o) qv[o] = int8_rne_sat(div_rn_recip(div_rn_recip(y[o], sm, rsm), p.scale, p.rscale));
        if (n == 4 && kBulk) {
          *reinterpret_cast<uint32_t*>(yrow_i + t) = static_cast<uint32_t>(static_cast<uint8_t>(qv[0])) |
                                                     static_cast<uint32_t>(static_cast<uint8_t>(qv[1])) << 8 |
                                                     static_cast<uint32_t>(static_cast<uint8_t>(qv[2])) << 16 |
                                                     static_cast<uint32_t>(static_cast<uint8_t>(qv[3])) << 24;
        } else {
#pragma unroll
          for (int o = 0; o < 4; ++o)
            if (o < n) yrow_i[t + o] = qv[o];
        }
      } else {
        if (n == 4 && kBulk) {
          *reinterpret_cast<float4*>(yrow_f + t) = make_float4(y[0], y[1], y[2], y[3]);   // 16-byte aligned
        } else {
#pragma unroll
          for (int o = 0; o < 4; ++o)
            if (o < n) yrow_f[t + o] = y[o];
        }
      }
    }
    __syncthreads();   // hs and this tile's xs buffer are free for reuse
  }
  // Drain: no bulk copy may still be writing this block's shared memory at exit.
  if (kBulk && tid == 0) {
    if (pending0) fir_wait(&bar[0], phase0);
    if (pending1) fir_wait(&bar[1], phase1);
  }
}

}  // namespace isp
