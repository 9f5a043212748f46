// Small-M (decode) W8A8 GEMM: out[M <= 128, N] = epilogue(A . W^T), K split
// across a thread-block cluster, partial sums reduced through distributed
// shared memory.  Decode is bound by streaming the weight once from HBM; with
// one 128 x 256 tile per CTA the regular kernel would run only N/256 CTAs, each
// reading a whole K row block of W and all of A.  Here a cluster of S CTAs
// shares one 128-column N tile:
//   * CTA r of the cluster runs the TMA -> tcgen05 main loop over K blocks
//     [r kb/S, (r+1) kb/S) into one TMEM accumulator (128 lanes x 128 columns),
//     then writes its partial (rows < M) to its own shared memory;
//   * after a cluster barrier, CTA r sums the S partials of its 128/S output
//     columns (peer shared memory via ld.shared::cluster, fixed order q = 0..S-1)
//     and applies the epilogue of the regular kernel (scale, bias, residual);
//   * a second cluster barrier keeps every CTA's shared memory alive until all
//     readers are done.
// No global workspace, one launch.  Every CTA reaches both cluster barriers on
// every path (including expired waits), so a peer can never be left waiting.
// INT8 partial sums are int32 and add exactly; FP8 partial sums are FP32 and
// add in the fixed rank order (deterministic, rounding order differs from the
// single-CTA kernel by the split).
#pragma once

#include "gemm_sm100.cuh"

namespace isp {
namespace gemm {

constexpr int kDecBN = 128;
constexpr int kDecStages = 6;            // up to 6 K blocks per CTA: every weight tile is requested before the wait
constexpr int kDecMaxSplits = 8;
constexpr int kDecThreads = 192;          // warp 0 TMA, warp 1 MMA, warps 2-5 TMEM -> shared
constexpr int kDecRowStride = 528;        // bytes per partial row: 128 x 4 B + 16 B (conflict-free 16-byte stores)

struct DecSmem {
  static constexpr int kABytes = kBM * kBK;        // 16 KB
  static constexpr int kBBytes = kDecBN * kBK;     // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  // The partial sums reuse the stage buffers: they are written after the CTA's
  // last MMA has completed, and with it every TMA load those MMAs consumed.
  static constexpr int kRedOffset = 0;
  static constexpr int kRedBytes = kBM * kDecRowStride;
  // Epilogue operands staged in shared memory: w_scale and bias of the tile's
  // columns (read before the programmatic-dependency wait), the scale of each row.
  static constexpr int kParamOffset = kDecStages * kStageBytes;
  static constexpr int kParamBytes = (2 * kDecBN + kBM) * 4;
  static constexpr int kBarOffset = kParamOffset + kParamBytes;
  static constexpr int kBytes = kBarOffset + 128;
  static_assert(kRedBytes <= kDecStages * kStageBytes, "partials must fit in the stage buffers");
};

// cluster_rank, cluster_sync_all and map_to_rank are in gemm_sm100.cuh
ISP_D uint4 ld_cluster_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <bool kInt8>
ISP_D float dec_acc(uint32_t bits) {
  if constexpr (kInt8) return static_cast<float>(static_cast<int32_t>(bits));
  else return __uint_as_float(bits);
}

// The regular kernel's EPI_SCALE arithmetic for one value (see scale_group).
template <bool kInt8>
ISP_D float dec_scale(float acc, const Params& p, float sa, float ws, float b) {
  if (p.a_scale_rows != nullptr) {
    if constexpr (kInt8) return __fadd_rn(__fmul_rn(acc, __fmul_rn(sa, ws)), b);
    else return __fmaf_rn(__fmul_rn(acc, sa), ws, b);
  }
  const float c = __fmul_rn(p.a_scale, ws);
  if constexpr (kInt8) return __fadd_rn(__fmul_rn(acc, c), b);
  else return __fmaf_rn(acc, c, b);
}

template <bool kInt8, int kOut>
__global__ void __launch_bounds__(kDecThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, const Params p,
                  int splits) {
  using L = DecSmem;
  extern __shared__ __align__(1024) uint8_t smem[];
  // A misaligned base skips the work but still takes part in both cluster barriers.
  const bool aligned = (smem_u32(smem) & 1023u) == 0;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty_bar = full_bar + kDecStages;
  uint64_t* tfull_bar = empty_bar + kDecStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint8_t* red = smem + L::kRedOffset;
  float* ws_s = reinterpret_cast<float*>(smem + L::kParamOffset);
  float* bias_s = ws_s + kDecBN;
  float* sa_s = bias_s + kDecBN;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_rank());
  const int n0 = blockIdx.y * kDecBN;
  const int kb0 = static_cast<int>(static_cast<int64_t>(rank) * p.k_blocks / splits);
  const int kb1 = static_cast<int>(static_cast<int64_t>(rank + 1) * p.k_blocks / splits);

  if (threadIdx.x == 0) {
    if (!aligned) atomicExch(&g_device_error, (int)ISP_ERR_ALIGN);
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tfull_bar, 1);
    *abort_flag = aligned ? 0 : 1;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tmap(&tm_a);
    prefetch_tmap(&tm_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kDecBN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const bool run = aligned;
  // The weight does not depend on the preceding kernel: the producer streams the
  // weight tiles of its first stages before waiting for it, so this launch's HBM
  // reads overlap the predecessor's tail; A (its output) is loaded after the wait.
  const int npre = run ? min(kDecStages, kb1 - kb0) : 0;
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < npre; ++i) {
      uint8_t* sa = smem + i * L::kStageBytes;
      mbar_expect_tx(&full_bar[i], L::kStageBytes);
      tma_load_2d(sa + L::kABytes, &tm_b, &full_bar[i], (kb0 + i) * kBK, n0);
    }
  }
  if (warp >= 2) {   // per-column weight scale and bias: weights, like the tiles above
    const int c = threadIdx.x - 64;
    const int n = n0 + c;
    ws_s[c] = (p.w_scale != nullptr && n < p.N) ? __ldg(p.w_scale + n) : 1.f;
    bias_s[c] = (p.bias != nullptr && n < p.N) ? __ldg(p.bias + n) : 0.f;
  }
  pdl_wait();      // predecessor complete before any activation or output access
  pdl_trigger();
  if (warp >= 2) {
    const int m = threadIdx.x - 64;
    sa_s[m] = p.a_scale_rows != nullptr ? (m < p.M ? __ldg(p.a_scale_rows + m) : 0.f) : p.a_scale;
  }

  if (warp == 0 && run) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool armed[kDecStages];
    uint32_t armed_phase[kDecStages];
#pragma unroll
    for (int s = 0; s < kDecStages; ++s) {
      armed[s] = false;
      armed_phase[s] = 0;
    }
    for (int kb = kb0; kb < kb1; ++kb) {
      const bool pre = kb - kb0 < npre;       // stage armed and its weight tile issued above
      if (!pre && !wait_warp(&empty_bar[stage], phase ^ 1u, abort_flag)) break;
      armed[stage] = true;
      armed_phase[stage] = phase;
      if (lane == 0) {
        uint8_t* sa = smem + stage * L::kStageBytes;
        if (!pre) mbar_expect_tx(&full_bar[stage], L::kStageBytes);
        tma_load_2d(sa, &tm_a, &full_bar[stage], kb * kBK, 0);
        if (!pre) tma_load_2d(sa + L::kABytes, &tm_b, &full_bar[stage], kb * kBK, n0);
      }
      __syncwarp();
      if (++stage == kDecStages) { stage = 0; phase ^= 1u; }
    }
    for (int s = 0; s < kDecStages; ++s)            // in-flight loads land before the CTA exits
      if (armed[s]) wait_warp_drain(&full_bar[s], armed_phase[s]);
  } else if (warp == 1 && run) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = instr_desc<kInt8 ? AB_I8 : AB_E4M3, kDecBN>();
    int stage = 0;
    uint32_t phase = 0;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!wait_warp(&full_bar[stage], phase, abort_flag)) break;
      tc_fence_after();
      {   // the whole warp: operands computed warp-wide, one elected lane issues
        const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
        const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 32; ++kk)
          mma_issue_elect<kInt8, false>(tmem_base, smem_desc_sw128(a_addr + kk * 32),
                                        smem_desc_sw128(b_addr + kk * 32), idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        mma_commit_elect<false>(&empty_bar[stage]);
      }
      __syncwarp();
      if (++stage == kDecStages) { stage = 0; phase ^= 1u; }
    }
    if (lane == 0) mma_commit(tfull_bar);    // also the drain: arrives once every issued MMA completed
    __syncwarp();
    wait_warp_drain(tfull_bar, 0);           // (also on abort: TMEM is freed only after it)
  } else if (warp >= 2 && run) {
    // ------------------------------------------------ TMEM -> shared partial
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool have = kb1 > kb0;
    if (wait_bounded(tfull_bar, 0, abort_flag)) {
      tc_fence_after();
      uint8_t* dst = red + row * kDecRowStride;
#pragma unroll
      for (int g = 0; g < kDecBN / 32; ++g) {
        uint32_t r[32];
        tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + g * 32, r);
        tmem_ld_wait(r);
        if (row < p.M) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 v = have ? make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]) : make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(dst + (g * 32 + 4 * j) * 4) = v;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();    // every partial of the cluster is in shared memory

  // ------------------------------------------- cluster reduction + epilogue
  if (run) {
    const int cols = kDecBN / splits;          // this CTA's output columns
    const int c0 = rank * cols;
    const int vec_per_row = cols / 4;
    const int items = p.M * vec_per_row;
    for (int i = threadIdx.x; i < items; i += kDecThreads) {
      const int m = i / vec_per_row;
      const int c = c0 + 4 * (i - m * vec_per_row);
      const int n = n0 + c;
      if (n >= p.N) continue;                  // N % 16 == 0: a 4-column group is wholly in or out
      const uint32_t local = smem_u32(red + m * kDecRowStride + c * 4);
      // all of the cluster's partials of this group requested before the first is used
      uint4 t[kDecMaxSplits];
#pragma unroll
      for (int q = 0; q < kDecMaxSplits; ++q)
        if (q < splits) t[q] = ld_cluster_v4(map_to_rank(local, q));
      float v[4];
      if constexpr (kInt8) {
        int32_t s4[4] = {0, 0, 0, 0};
#pragma unroll
        for (int q = 0; q < kDecMaxSplits; ++q) {
          if (q < splits) {
            s4[0] += static_cast<int32_t>(t[q].x); s4[1] += static_cast<int32_t>(t[q].y);
            s4[2] += static_cast<int32_t>(t[q].z); s4[3] += static_cast<int32_t>(t[q].w);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = static_cast<float>(s4[j]);
      } else {
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < kDecMaxSplits; ++q) {
          if (q < splits) {
            s4[0] = __fadd_rn(s4[0], __uint_as_float(t[q].x)); s4[1] = __fadd_rn(s4[1], __uint_as_float(t[q].y));
            s4[2] = __fadd_rn(s4[2], __uint_as_float(t[q].z)); s4[3] = __fadd_rn(s4[3], __uint_as_float(t[q].w));
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = s4[j];
      }
      const float sa = sa_s[m];
      const int64_t off = static_cast<int64_t>(m) * p.N + n;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[j] = dec_scale<kInt8>(v[j], p, sa, ws_s[c + j], bias_s[c + j]);
        if (p.residual != nullptr) {
          const float r = p.residual_f32 ? __ldg(static_cast<const float*>(p.residual) + off + j)
                                         : __bfloat162float(static_cast<const __nv_bfloat16*>(p.residual)[off + j]);
          v[j] = __fadd_rn(v[j], r);
        }
      }
      if constexpr (kOut == OUT_F32) {
        *reinterpret_cast<float4*>(static_cast<float*>(p.out) + off) = make_float4(v[0], v[1], v[2], v[3]);
      } else if constexpr (kOut == OUT_BF16) {
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + off) =
            make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
      } else {
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.out) + off) =
            make_uint2(pack_f16(v[0], v[1]), pack_f16(v[2], v[3]));
      }
    }
  }
  cluster_sync_all();    // no CTA leaves while a peer may still read its shared memory

  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kDecBN));
  }
}

}  // namespace gemm
}  // namespace isp
