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

// ---------------------------------------------------------------- GEMV (M = 1)
// Weight-streaming GEMV: one CTA per SM owns a contiguous range of output columns, whose packed
// weights are one contiguous byte range of the image ([N][K/2]). Each of 12 warps takes every 12th
// column of the range; a column's K words (16 bytes = 32 values) are spread over the lanes, each
// word is 8 dp4a on 16 * w and the activations, shifted by the group's exponent, and a warp
// reduction ends the column with its SRS. The weights are read straight from global memory with
// 16-byte streaming loads, all of a batch's loads (CPB columns x WPL words per lane, up to 8)
// issued before any is used. One CTA per SM at half the SM's registers, launched with
// programmatic dependent launch: it lets the next kernel on the stream launch at once, and the
// next GEMV of a chain (a decode step's layers) then sits beside it on the same SM and asks for
// its own weight range in the L2 (a bulk prefetch, a hint that reads nothing it depends on) while
// this one streams; it waits for the previous kernel (griddepcontrol.wait) before any load whose
// value it uses, then stages the activations and the CTA's group exponents in shared memory.
constexpr int kGemvWarps = 12;
constexpr int kGemvThreads = 32 * kGemvWarps;
constexpr int kGemvMaxWpl = 8;           // 16-byte loads per lane in flight per batch
constexpr int kGemvCtasPerSm = 2;        // for the registers: this GEMV and the next

struct GemvPlan {
  int grid, wpl, eg_bytes, smem;
};

__host__ inline GemvPlan plan_gemv(int N, int K, int sms) {
  GemvPlan g;
  g.grid = std::min(sms, N);
  const int words = K / 32;
  g.wpl = std::min(kGemvMaxWpl, (words + 31) / 32);  // columns of more words are taken in segments
  // the group exponents of a CTA's columns (at most ceil(N / grid) of them), from the 16-byte
  // boundary at or below the first to the one at or above the last (up to 15 more on each side)
  g.eg_bytes = ((N + g.grid - 1) / g.grid * (K / kW4Group) + 32 + 15) / 16 * 16;
  g.smem = K + g.eg_bytes;
  return g;
}

__device__ __forceinline__ uint4 ld_stream16(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16 * sum over one 16-byte word (32 values) of a * w, shifted down by the group exponent e:
// exact, the dp4a sum being a multiple of 16.
__device__ __forceinline__ int gemv_word(uint4 w, const int8_t* a_s, int wd, uint32_t e) {
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
  return pr >> e;
}

// One warp's columns, CPB at a time, WPL words per lane per column (the column's words wd = lane +
// 32 i); columns of more than 32 * WPL words go in segments of 32 * WPL words.
template <int WPL>
__device__ __forceinline__ void gemv_warp(const uint8_t* __restrict__ wq, const int32_t* __restrict__ shift,
                                          int8_t* __restrict__ out, const int8_t* a_s, const uint8_t* eg_s,
                                          long long e_lo, int n0, int n1, int K, int warp, int lane) {
  constexpr int CPB = kGemvMaxWpl / WPL > 4 ? 4 : kGemvMaxWpl / WPL;
  const int words = K / 32, G = K / kW4Group, col_bytes = K / 2;
  for (int t0 = 0;; t0 += CPB) {
    int col[CPB];
    bool any = false;
#pragma unroll
    for (int j = 0; j < CPB; ++j) {
      col[j] = n0 + warp + kGemvWarps * (t0 + j);
      any |= col[j] < n1;
    }
    if (!any) break;
    int acc[CPB];
#pragma unroll
    for (int j = 0; j < CPB; ++j) acc[j] = 0;
    for (int seg = 0; seg < words; seg += 32 * WPL) {
      uint4 w[CPB][WPL];
#pragma unroll
      for (int j = 0; j < CPB; ++j) {
        const uint8_t* cw = wq + (long long)col[j] * col_bytes + (seg + lane) * 16;  // word seg + lane of column j
#pragma unroll
        for (int i = 0; i < WPL; ++i)
          if (col[j] < n1 && seg + i * 32 + lane < words) w[j][i] = ld_stream16(cw + i * 512);
      }
#pragma unroll
      for (int j = 0; j < CPB; ++j) {
        const uint8_t* erow = eg_s + ((long long)col[j] * G - e_lo);
#pragma unroll
        for (int i = 0; i < WPL; ++i) {
          const int wd = seg + i * 32 + lane;
          if (col[j] < n1 && wd < words) acc[j] += gemv_word(w[j][i], a_s, wd, erow[wd >> 2]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < CPB; ++j) {
      int v = acc[j];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && col[j] < n1) out[col[j]] = (int8_t)clamp_i8(rne_shift(v, __ldg(shift + col[j])));
    }
  }
}

template <int WPL>
__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm)
    w4a8_gemv_kernel(const int8_t* __restrict__ a, const uint8_t* __restrict__ wq, const uint8_t* __restrict__ eg,
                     const int32_t* __restrict__ shift, int8_t* __restrict__ out, int N, int K) {
  extern __shared__ __align__(16) uint8_t gsm[];
  int8_t* a_s = reinterpret_cast<int8_t*>(gsm);  // [K]
  uint8_t* eg_s = gsm + K;                        // exponents [e_lo, e_hi) of [N][K / 128]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = (int)((long long)blockIdx.x * N / gridDim.x), n1 = (int)((long long)(blockIdx.x + 1) * N / gridDim.x);
  const int G = K / kW4Group;
  // the CTA's exponents [n0, n1) x G are one contiguous run of [N][K / 128]; the staged range starts
  // at the 16-byte boundary below it and ends at the one above (N * G is a multiple of 16: N is)
  const long long e_lo = ((long long)n0 * G) & ~15LL, e_hi = ((long long)n1 * G + 15) & ~15LL;
  grid_dep_launch();  // the next kernel may launch; it waits for this one before using any result
  if (tid == 0) {
    const long long w0 = (long long)n0 * (K / 2), w1 = (long long)n1 * (K / 2);  // 16-byte multiples
    for (long long off = w0; off < w1; off += 65536)
      bulk_prefetch_l2(wq + off, (uint32_t)(w1 - off < 65536 ? w1 - off : 65536));
    bulk_prefetch_l2(eg + e_lo, (uint32_t)(e_hi - e_lo));
  }
  grid_dep_wait();  // the activations, and anything the previous kernel wrote, from here on
  for (int i = tid; i < K / 16; i += kGemvThreads)
    reinterpret_cast<int4*>(a_s)[i] = __ldg(reinterpret_cast<const int4*>(a) + i);
  for (long long i = e_lo / 16 + tid; i < e_hi / 16; i += kGemvThreads)
    reinterpret_cast<uint4*>(eg_s)[i - e_lo / 16] = __ldg(reinterpret_cast<const uint4*>(eg) + i);
  __syncthreads();
  gemv_warp<WPL>(wq, shift, out, a_s, eg_s, e_lo, n0, n1, K, warp, lane);
}

}  // namespace ixb
