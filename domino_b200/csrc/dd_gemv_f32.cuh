// dd_gemv_f32.cuh -- the contractions of the draft step for fp32 heads.
//
// The reference runs an fp32 draft head (its CPU-runnable configuration, and
// any fp32 checkpoint) with fp32 arithmetic throughout: fp32 F.linear for the
// z / s / gh projections, the W_ih table and lm_head, and fp32 FMA for the
// fused correction step (code/kernel/domino.py:58-136, 374-431).  bf16 tensor
// cores cannot reproduce that, so fp32 heads stream their fp32 weights through
// this CUDA-core kernel instead: every product is an fp32 FMA.  At the batch
// sizes of the draft step the contraction is HBM-bound (one FMA per 4-byte
// weight per batch row), so the CUDA cores are not the limit.
//
// Layout: a CTA of 8 warps owns 32 consecutive weight rows (4 per warp) and
// walks K in chunks of 512; each chunk of the X rows (at most 16 per launch)
// is staged once in shared memory and read as float4 by every warp.  Each lane
// accumulates its share of K for (4 rows x 16 X rows); a warp reduction then
// leaves lane j holding the 4 row results of X row j, which it hands to the
// phase's epilogue (the same kinds as the tensor-core kernel, in fp32).
#pragma once

#include "dd_gemv.cuh"

namespace dd {

constexpr int kF32Threads = 256;
constexpr int kF32Warps = kF32Threads / 32;
constexpr int kF32RowsPerWarp = 4;
constexpr int kF32RowsPerCta = kF32Warps * kF32RowsPerWarp;  // 32
constexpr int kF32KChunk = 512;                               // X columns staged per round
constexpr int kF32MaxN = 16;                                  // X rows per launch

template <int kPhase>
__device__ __forceinline__ void epilogue_f32(const GemvParams& p, int kind, int row, long long gn, float v) {
  if (phase_has<kPhase>(EPI_ZPROJ) && kind == EPI_ZPROJ) {
    const float bias = p.fc1_bias ? static_cast<const float*>(p.fc1_bias)[row] : 0.0f;
    static_cast<float*>(p.z_out)[gn * p.E + row] = v + bias;
  } else if (phase_has<kPhase>(EPI_LMHEAD) && kind == EPI_LMHEAD) {
    static_cast<float*>(p.base_out)[gn * p.base_out_ld + row] = v;
  } else if (phase_has<kPhase>(EPI_TABLE) && kind == EPI_TABLE) {
    const float bias = p.b_ih ? static_cast<const float*>(p.b_ih)[row] : 0.0f;
    static_cast<float*>(p.table_out)[gn * p.table_ld + row] = v + bias;
  } else if (phase_has<kPhase>(EPI_GH) && kind == EPI_GH) {
    const float bias = p.b_hh ? static_cast<const float*>(p.b_hh)[row] : 0.0f;
    static_cast<float*>(p.gh_out)[gn * p.G3 + row] = v + bias;
  } else if (phase_has<kPhase>(EPI_SPROJ_MID) && kind == EPI_SPROJ_MID) {
    // s = h W_s^T (fp32, domino.py:397); mid = middle(z_t + s) (domino.py:95-96, 406-408)
    if (p.s_out) static_cast<float*>(p.s_out)[gn * p.E + row] = v;
    const size_t zrow = (size_t)gn * p.z_rows_per_b + p.z_pos_off + p.t;
    const float pre = static_cast<const float*>(p.z_src)[zrow * p.E + row] + v;
    static_cast<float*>(p.mid_out)[gn * p.E + row] = middle_act(p.middle, pre);
  }
}

template <int kPhase>
__global__ void __launch_bounds__(kF32Threads) gemv_f32_kernel(const GemvParams p) {
  __shared__ __align__(16) float xs[kF32MaxN * kF32KChunk];  // 32 KB
  __shared__ unsigned long long red[kF32Warps][kF32MaxN];
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = p.n_valid;  // X rows of this launch, <= kF32MaxN
  const int K = p.K;

  // This warp's rows: global index g over the segments (seg 0 rows, then seg 1).
  const long long g0 = (long long)blockIdx.x * kF32RowsPerCta + warp * kF32RowsPerWarp;
  const float* wrow[kF32RowsPerWarp];
  int row[kF32RowsPerWarp], kind[kF32RowsPerWarp];
  bool rvalid[kF32RowsPerWarp];
#pragma unroll
  for (int i = 0; i < kF32RowsPerWarp; ++i) {
    const long long g = g0 + i;
    const int s = g >= p.seg[0].rows ? 1 : 0;
    const long long local = s ? g - p.seg[0].rows : g;
    rvalid[i] = s == 0 || (p.nseg > 1 && local < p.seg[1].rows);
    row[i] = p.seg[s].row_off + (int)local;
    kind[i] = p.seg[s].kind;
    wrow[i] = rvalid[i] ? p.w32[s] + (size_t)row[i] * p.w32_ld[s] : nullptr;
  }

  float acc[kF32RowsPerWarp][kF32MaxN];
#pragma unroll
  for (int i = 0; i < kF32RowsPerWarp; ++i)
#pragma unroll
    for (int j = 0; j < kF32MaxN; ++j) acc[i][j] = 0.0f;

  pdl_wait_primary();  // X comes from the previous kernel
  for (int k0 = 0; k0 < K; k0 += kF32KChunk) {
    const int kc4 = min(kF32KChunk, K - k0) / 4;  // K is a multiple of 8
    for (int i = threadIdx.x; i < n * kc4; i += kF32Threads) {
      const int j = i / kc4, c = i - j * kc4;
      reinterpret_cast<float4*>(xs + j * kF32KChunk)[c] =
          reinterpret_cast<const float4*>(p.x32 + (size_t)(p.n_off + j) * p.x32_ld + k0)[c];
    }
    __syncthreads();
    for (int c = lane; c < kc4; c += 32) {
      float4 wv[kF32RowsPerWarp];
#pragma unroll
      for (int i = 0; i < kF32RowsPerWarp; ++i)
        wv[i] = rvalid[i] ? __ldcs(reinterpret_cast<const float4*>(wrow[i] + k0) + c) : make_float4(0, 0, 0, 0);
#pragma unroll
      for (int j = 0; j < kF32MaxN; ++j) {
        if (j < n) {
          const float4 xv = reinterpret_cast<const float4*>(xs + j * kF32KChunk)[c];
#pragma unroll
          for (int i = 0; i < kF32RowsPerWarp; ++i) {
            acc[i][j] = fmaf(wv[i].x, xv.x, acc[i][j]);
            acc[i][j] = fmaf(wv[i].y, xv.y, acc[i][j]);
            acc[i][j] = fmaf(wv[i].z, xv.z, acc[i][j]);
            acc[i][j] = fmaf(wv[i].w, xv.w, acc[i][j]);
          }
        }
      }
    }
    __syncthreads();
  }

  // Warp sums: lane j keeps the results of X row j.
  float out[kF32RowsPerWarp];
#pragma unroll
  for (int i = 0; i < kF32RowsPerWarp; ++i) {
    out[i] = 0.0f;
#pragma unroll
    for (int j = 0; j < kF32MaxN; ++j) {
      if (j < n) {
        float v = acc[i][j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
        if (lane == j) out[i] = v;
      }
    }
  }

  const bool has_argmax = (phase_has<kPhase>(EPI_FC2_ARGMAX) || phase_has<kPhase>(EPI_LMHEAD));
  unsigned long long key = 0ull;  // lane j: best (logit, index) word of X row j over this warp's rows
  if (lane < n) {
    const long long gn = p.n_off + lane;
#pragma unroll
    for (int i = 0; i < kF32RowsPerWarp; ++i) {
      if (!rvalid[i]) continue;
      if (phase_has<kPhase>(EPI_FC2_ARGMAX) && kind[i] == EPI_FC2_ARGMAX) {
        // logit = mid . fc2[v] + fc2_bias[v] + base_t[v] (domino.py:126-136)
        float logit = out[i];
        if (p.fc2_bias) logit += static_cast<const float*>(p.fc2_bias)[row[i]];
        const size_t brow = (size_t)gn * p.base_rows_per_b + p.base_pos_off + p.t;
        logit += static_cast<const float*>(p.base_src)[brow * p.base_ld + p.base_voff + row[i]];
        const unsigned long long k = argmax_key(logit, (uint32_t)(p.v_off + row[i]));
        key = k > key ? k : key;
      } else {
        epilogue_f32<kPhase>(p, kind[i], row[i], gn, out[i]);
        if (phase_has<kPhase>(EPI_LMHEAD) && kind[i] == EPI_LMHEAD && (int)(gn % p.kpos) < p.npre) {
          const unsigned long long k = argmax_key(out[i], (uint32_t)(p.v_off + row[i]));
          key = k > key ? k : key;
        }
      }
    }
  }
  if (has_argmax) {
    if (lane < kF32MaxN) red[warp][lane] = key;
    __syncthreads();
    if ((int)threadIdx.x < n) {
      const int j = threadIdx.x;
      unsigned long long k = red[0][j];
#pragma unroll
      for (int w = 1; w < kF32Warps; ++w) k = red[w][j] > k ? red[w][j] : k;
      if (k) {
        const long long gn = p.n_off + j;
        if (phase_has<kPhase>(EPI_FC2_ARGMAX) && kPhase == PH_FC2) {
          atomicMax(p.slots + (size_t)gn * p.nslots + p.npre + p.t, k);
        } else if ((int)(gn % p.kpos) < p.npre) {
          atomicMax(p.slots + (size_t)(gn / p.kpos) * p.nslots + (int)(gn % p.kpos), k);
        }
      }
    }
  }
}

}  // namespace dd
