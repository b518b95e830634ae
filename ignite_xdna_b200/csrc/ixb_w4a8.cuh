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
// One warp per output column; the lanes split K (32 values per lane per step, a step covers 1024)
// and the column's partial sums meet in a warp reduction. Weights stream once from HBM; the
// activation vector stays in L1.
__global__ void __launch_bounds__(256) w4a8_gemv_kernel(const int8_t* __restrict__ a, const uint8_t* __restrict__ wq,
                                                        const uint8_t* __restrict__ eg,
                                                        const int32_t* __restrict__ shift, int8_t* __restrict__ out,
                                                        int N, int K) {
  const int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  const uint8_t* row = wq + (long long)n * (K / 2);
  const uint8_t* erow = eg + (long long)n * (K / kW4Group);
  int acc = 0;
  // all of a lane's weight loads (up to 8 x 16 bytes) are in flight before the first is used
  constexpr int kBatch = 8;
  for (int kb = lane * 32; kb < K; kb += 1024 * kBatch) {
    uint4 w[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int k0 = kb + j * 1024;
      if (k0 < K)
        asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(w[j].x), "=r"(w[j].y), "=r"(w[j].z), "=r"(w[j].w)
                     : "l"(row + k0 / 2));
      else
        w[j] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      const int k0 = kb + j * 1024;
      if (k0 >= K) break;
      const int4 a0 = __ldg(reinterpret_cast<const int4*>(a + k0));
      const int4 a1 = __ldg(reinterpret_cast<const int4*>(a + k0) + 1);
      int p = 0;
      p = __dp4a((int)w4_lo16(w[j].x), a0.x, p);
      p = __dp4a((int)w4_hi16(w[j].x), a0.y, p);
      p = __dp4a((int)w4_lo16(w[j].y), a0.z, p);
      p = __dp4a((int)w4_hi16(w[j].y), a0.w, p);
      p = __dp4a((int)w4_lo16(w[j].z), a1.x, p);
      p = __dp4a((int)w4_hi16(w[j].z), a1.y, p);
      p = __dp4a((int)w4_lo16(w[j].w), a1.z, p);
      p = __dp4a((int)w4_hi16(w[j].w), a1.w, p);
      acc += p >> __ldg(erow + (k0 >> 7));  // p = 16 * sum a * w, a multiple of 16: exact
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[n] = (int8_t)clamp_i8(rne_shift(acc, __ldg(shift + n)));
}

}  // namespace ixb
