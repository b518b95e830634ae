// W4A8: int8 activations x packed int4 weights with per-group pow2 scales, int32 accumulation,
// per-output-channel pow2 SRS to int8.
//
// Reference operand format (kernels/w4a8_probe/w4a8_probe.py:197-201, tools/int4_prefill_model.py
// Int4WeightPacker / Int4MmulReference): B int4 [K][N] packed two per byte along N, element 2j in
// the low nibble, two's complement. The reference kernels (kernels/w4a8_probe/w4a8_kernels.cc,
// mm_i8i4_*) produce raw int32 C = A.B and have no group-scale step; the group rule here is this
// engine's own: with p_g,n the position (log2 of the scale's inverse) of group g of column n and
// d = max_g p_g,n - p_g,n,
//     acc[m][n] = sum_g (sum_{k in g} a[m][k] * w[k][n]) << d_g,n,
//     out[m][n] = clamp(rne(acc[m][n] >> shift[n]), -128, 127).
// Groups are 128 along K. Each d must lie in [0, 4]: then w << d fits int8 exactly, and the
// tensor cores (prefill) and dp4a (GEMV) accumulate the shifted products exactly in int32.
//
// ixb_w4a8_prepare converts the reference operand once into the engine's weight image:
//   wq  uint8 [N][K/2]: row n holds column n K-major; in each 4-byte word (8 values of k0..k0+7)
//                       byte j = nibble(k0 + j) | nibble(k0 + j + 4) << 4, so masking the word
//                       with 0xF0F0F0F0 after and before a 4-bit left shift yields k0..k3 and
//                       k4..k7 as int8 lanes holding 16 * w;
//   eg  uint8 [N][K/128]: e = 4 - d per (column, group); 16 * w >> e = w << d.
#pragma once
#include <cstdint>
#include <algorithm>
#include "ixb_ptx.cuh"

namespace ixb {

constexpr int kW4Group = 128;

// ---------------------------------------------------------------- weight image
__global__ void w4a8_pack_kernel(const uint8_t* __restrict__ w_kn, int K, int N, uint8_t* __restrict__ wq) {
  // thread per (column n, 8-value word w); consecutive threads take consecutive columns so the
  // reads of one reference row are coalesced
  const long long words = (long long)N * (K / 8);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < words;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const int w = (int)(i / N);
    const int k0 = 8 * w;
    uint32_t out = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint8_t byte = __ldg(w_kn + (long long)(k0 + j) * (N / 2) + (n >> 1));
      const uint32_t nib = (n & 1) ? (byte >> 4) : (byte & 0xFu);
      out |= nib << (j < 4 ? 8 * j : 8 * (j - 4) + 4);
    }
    *reinterpret_cast<uint32_t*>(wq + (long long)n * (K / 2) + 4 * w) = out;
  }
}

__global__ void w4a8_groups_kernel(const int8_t* __restrict__ gpos, int G, int N, uint8_t* __restrict__ eg) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  int pmax = -128;
  for (int g = 0; g < G; ++g) pmax = max(pmax, (int)gpos[(long long)g * N + n]);
  for (int g = 0; g < G; ++g) {
    const int d = pmax - (int)gpos[(long long)g * N + n];
    if (d > 4) set_dev_error(DEV_ERR_BAD_ARGS);
    eg[(long long)n * G + g] = (uint8_t)(4 - min(d, 4));
  }
}

// 16 * w as int8 lanes from one packed word: lanes k0..k3 and k4..k7.
__device__ __forceinline__ uint32_t w4_lo16(uint32_t x) { return (x << 4) & 0xF0F0F0F0u; }
__device__ __forceinline__ uint32_t w4_hi16(uint32_t x) { return x & 0xF0F0F0F0u; }

// Per-byte arithmetic shift right by e in [0, 4] of int8 lanes that are multiples of 16 (exact).
__device__ __forceinline__ uint32_t sra8_lanes(uint32_t v, uint32_t e, uint32_t keep, uint32_t fill) {
  // logical shift (low nibbles are zero, so no bits cross lanes), then the sign into the top e bits
  const uint32_t t = (v >> e) & keep;
  const uint32_t neg = (v >> 7) & 0x01010101u;
  return t + neg * fill;
}

// ---------------------------------------------------------------- GEMV (M = 1)
// Weight-streaming GEMV: one CTA per SM owns a contiguous range of output columns, whose packed
// weights are one contiguous byte range of the image ([N][K/2]). A producer thread streams that
// range through a ring of shared-memory stages with bulk copies (the TMA engine keeps up to
// ~200 KB per SM in flight, enough to cover DRAM latency at full bandwidth), while 16 consumer
// warps take the columns of each stage: a column's K words (16 bytes = 32 values) are split over
// the lanes (and, for large K, over several warps), each word is 8 dp4a on 16 * w and the
// activations (staged in shared memory once per CTA), shifted per group, and the partial sums
// meet in a warp (then a shared-memory) reduction before the per-column SRS.
constexpr int kGemvWarps = 16;                 // consumer warps
constexpr int kGemvThreads = 32 * (kGemvWarps + 1);
constexpr int kGemvSmemBudget = 200 * 1024;    // stages + activations

struct GemvPlan {
  int grid, cols_per_stage, warps_per_col, stages, stage_bytes, eg_bytes, smem;
};

__host__ inline GemvPlan plan_gemv(int N, int K, int sms) {
  GemvPlan g;
  const int col_bytes = K / 2;
  g.grid = std::min(sms, N);
  // the group exponents of a CTA's columns (at most ceil(N / grid) of them), staged once
  g.eg_bytes = ((N + g.grid - 1) / g.grid * (K / kW4Group) + 15) / 16 * 16;
  // columns per stage: 16 (one per warp) unless a stage would pass 96 KB or fewer than two fit
  for (int ch = kGemvWarps;; ch >>= 1) {
    g.cols_per_stage = ch;
    g.warps_per_col = kGemvWarps / ch;
    g.stage_bytes = ch * col_bytes;
    g.stages = std::min(4, (kGemvSmemBudget - K - g.eg_bytes) / g.stage_bytes);
    if (ch == 1 || (g.stage_bytes <= 96 * 1024 && g.stages >= 2)) break;
  }
  g.smem = g.stages * g.stage_bytes + K + g.eg_bytes + 2 * 8 * 4 + 1024;
  return g;
}

__global__ void __launch_bounds__(kGemvThreads, 1)
    w4a8_gemv_kernel(const int8_t* __restrict__ a, const uint8_t* __restrict__ wq, const uint8_t* __restrict__ eg,
                     const int32_t* __restrict__ shift, int8_t* __restrict__ out, int N, int K, int CH, int WPC,
                     int S, int stage_bytes, int eg_bytes) {
  extern __shared__ uint8_t gsm_raw[];
  uint8_t* gsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 127) & ~uintptr_t(127));
  uint8_t* eg_s = gsm + S * stage_bytes + K;   // [columns of this CTA][K / 128]
  uint64_t* full = reinterpret_cast<uint64_t*>(eg_s + eg_bytes);
  uint64_t* empty = full + 4;
  __shared__ int colsum[4][kGemvWarps], colcnt[4][kGemvWarps];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = (int)((long long)blockIdx.x * N / gridDim.x), n1 = (int)((long long)(blockIdx.x + 1) * N / gridDim.x);
  const int chunks = (n1 - n0 + CH - 1) / CH;
  const int col_bytes = K / 2, words = K / 32;
  int8_t* a_s = reinterpret_cast<int8_t*>(gsm + S * stage_bytes);
  if (tid == kGemvWarps * 32) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGemvWarps);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < K / 16; i += kGemvThreads)
    reinterpret_cast<int4*>(a_s)[i] = __ldg(reinterpret_cast<const int4*>(a) + i);
  {
    const int G = K / kW4Group;
    const long long e0 = (long long)n0 * G, e1 = (long long)n1 * G;  // contiguous: [N][K / 128]
    for (long long i = e0 + tid; i < e1; i += kGemvThreads) eg_s[i - e0] = __ldg(eg + i);
  }
  if (tid < 4 * kGemvWarps) {
    (&colsum[0][0])[tid] = 0;
    (&colcnt[0][0])[tid] = 0;
  }
  __syncthreads();
  if (warp == kGemvWarps) {
    // producer: chunk c (CH columns, the last one ragged) into stage c % S
    if (lane == 0) {
      uint32_t ph = 0;
      for (int c = 0, s = 0; c < chunks; ++c) {
        if (!mbar_wait(&empty[s], ph ^ 1)) break;
        const int cols = min(CH, n1 - n0 - c * CH);
        const uint32_t bytes = (uint32_t)cols * col_bytes;
        mbar_arrive_expect_tx(&full[s], bytes);
        const uint8_t* src = wq + ((long long)n0 + (long long)c * CH) * col_bytes;
        for (uint32_t off = 0; off < bytes; off += 32768u)
          bulk_g2s(gsm + s * stage_bytes + off, src + off, min(32768u, bytes - off), &full[s]);
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
    }
    return;
  }
  uint32_t ph = 0;
  const int G = K / kW4Group;
  for (int c = 0, s = 0; c < chunks; ++c) {
    const int cols = min(CH, n1 - n0 - c * CH);
    if (!mbar_wait(&full[s], ph)) break;
    const int ci = warp / WPC, part_i = warp % WPC;   // column of the chunk, share of its K words
    int acc = 0;
    if (ci < cols) {
      const int n = n0 + c * CH + ci;
      const uint8_t* col = gsm + s * stage_bytes + ci * col_bytes;
      const uint8_t* erow = eg_s + (n - n0) * G;
      for (int wd = part_i * 32 + lane; wd < words; wd += 32 * WPC) {
        const uint4 w = *reinterpret_cast<const uint4*>(col + wd * 16);
        const int4 a0 = reinterpret_cast<const int4*>(a_s)[2 * wd];
        const int4 a1 = reinterpret_cast<const int4*>(a_s)[2 * wd + 1];
        int pr = 0;
        pr = __dp4a((int)w4_lo16(w.x), a0.x, pr);
        pr = __dp4a((int)w4_hi16(w.x), a0.y, pr);
        pr = __dp4a((int)w4_lo16(w.y), a0.z, pr);
        pr = __dp4a((int)w4_hi16(w.y), a0.w, pr);
        pr = __dp4a((int)w4_lo16(w.z), a1.x, pr);
        pr = __dp4a((int)w4_hi16(w.z), a1.y, pr);
        pr = __dp4a((int)w4_lo16(w.w), a1.z, pr);
        pr = __dp4a((int)w4_hi16(w.w), a1.w, pr);
        acc += pr >> erow[wd >> 2];   // pr = 16 * sum a * w, a multiple of 16: exact
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    }
    if (lane == 0 && ci < cols) {
      const int n = n0 + c * CH + ci;
      if (WPC == 1) {
        out[n] = (int8_t)clamp_i8(rne_shift(acc, __ldg(shift + n)));
      } else {
        // the column's warps meet in shared memory: the last to arrive writes the output and
        // clears the slot, before its release of the stage lets the slot be used again
        atomicAdd(&colsum[s][ci], acc);
        __threadfence_block();
        if (atomicAdd(&colcnt[s][ci], 1) == WPC - 1) {
          __threadfence_block();
          const int sum = atomicExch(&colsum[s][ci], 0);
          colcnt[s][ci] = 0;
          out[n] = (int8_t)clamp_i8(rne_shift(sum, __ldg(shift + n)));
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);   // this warp is done with the stage
    if (++s == S) {
      s = 0;
      ph ^= 1;
    }
  }
}

}  // namespace ixb
