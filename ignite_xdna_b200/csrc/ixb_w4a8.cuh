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
// Weight-streaming GEMV: a warp per output column (or two short columns), eight warps per CTA
// (many small CTAs, four resident per SM, so DRAM latency hides behind other CTAs' loads); a column's K words
// (16 bytes = 32 values) are spread over the lanes, and all of a lane's loads of a batch (up to 8)
// are in flight before the first is used. Each word is 8 dp4a on 16 * w and the activations (read
// through L1), shifted by the group's exponent, and a warp reduction ends the column with its SRS.
// Launched with programmatic dependent launch: the kernel lets the next kernel on the stream
// launch at once, so in a chain of GEMVs (a decode step's layers) the next one's CTAs ask for
// their weight ranges in the L2 (a bulk prefetch: a hint, which reads nothing they use) while this
// one streams; every load whose value a CTA uses comes after it waits for the previous kernel
// (griddepcontrol.wait).
constexpr int kGemvWarps = 8;
constexpr int kGemvThreads = 32 * kGemvWarps;
constexpr int kGemvBatch = 8;           // 16-byte loads per lane in flight

__device__ __forceinline__ uint4 ld_stream16(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// CPW columns per warp: with K <= 4096 a column is at most four 16-byte loads per lane, so a warp
// takes two columns (kGemvWarps apart) and keeps eight loads in flight; the activations it reads
// once serve both. Longer columns take one column per warp and batches of eight loads.
template <int CPW>
__global__ void __launch_bounds__(kGemvThreads, 4)
    w4a8_gemv_kernel(const int8_t* __restrict__ a, const uint8_t* __restrict__ wq, const uint8_t* __restrict__ eg,
                     const int32_t* __restrict__ shift, int8_t* __restrict__ out, int N, int K) {
  constexpr int B = kGemvBatch / CPW;  // loads per column per batch
  const int n0 = blockIdx.x * kGemvWarps * CPW, warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int col_bytes = K / 2, G = K / kW4Group;
  grid_dep_launch();  // the next kernel may launch; it waits for this one before using any result
  if (threadIdx.x == 0) {
    const int cols = min(kGemvWarps * CPW, N - n0);  // the CTA's columns: one contiguous run of each table
    bulk_prefetch_l2(wq + (long long)n0 * col_bytes, (uint32_t)(cols * col_bytes));
    const long long e_lo = ((long long)n0 * G) & ~15LL, e_hi = ((long long)(n0 + cols) * G + 15) & ~15LL;
    bulk_prefetch_l2(eg + e_lo, (uint32_t)(e_hi - e_lo));
  }
  grid_dep_wait();  // the activations, and anything the previous kernel wrote, from here on
  int nc[CPW], acc[CPW];
  bool ok[CPW];
#pragma unroll
  for (int c = 0; c < CPW; ++c) {
    nc[c] = n0 + c * kGemvWarps + warp;
    ok[c] = nc[c] < N;  // warp-uniform
    acc[c] = 0;
  }
  if (!ok[0]) return;
  for (int k0 = lane * 32; k0 < K; k0 += 1024 * B) {
    uint4 w[CPW][B];
#pragma unroll
    for (int c = 0; c < CPW; ++c)
#pragma unroll
      for (int j = 0; j < B; ++j)
        if (ok[c] && k0 + j * 1024 < K) w[c][j] = ld_stream16(wq + (long long)nc[c] * col_bytes + (k0 + j * 1024) / 2);
#pragma unroll
    for (int j = 0; j < B; ++j) {
      const int k = k0 + j * 1024;
      if (k < K) {
        const int4 a0 = __ldg(reinterpret_cast<const int4*>(a + k));
        const int4 a1 = __ldg(reinterpret_cast<const int4*>(a + k) + 1);
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          if (!ok[c]) continue;
          int pr = 0;
          pr = __dp4a((int)w4_lo16(w[c][j].x), a0.x, pr);
          pr = __dp4a((int)w4_hi16(w[c][j].x), a0.y, pr);
          pr = __dp4a((int)w4_lo16(w[c][j].y), a0.z, pr);
          pr = __dp4a((int)w4_hi16(w[c][j].y), a0.w, pr);
          pr = __dp4a((int)w4_lo16(w[c][j].z), a1.x, pr);
          pr = __dp4a((int)w4_hi16(w[c][j].z), a1.y, pr);
          pr = __dp4a((int)w4_lo16(w[c][j].w), a1.z, pr);
          pr = __dp4a((int)w4_hi16(w[c][j].w), a1.w, pr);
          acc[c] += pr >> __ldg(eg + (long long)nc[c] * G + (k >> 7));  // pr = 16 * sum a * w: exact
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < CPW; ++c) {
    int v = acc[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && ok[c]) out[nc[c]] = (int8_t)clamp_i8(rne_shift(v, __ldg(shift + nc[c])));
  }
}

}  // namespace ixb
