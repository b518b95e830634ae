// Bandwidth-bound kernels of the XINT8 graph: image ingress (pixel -> int8 lookup into the
// padded 8-byte-pixel stem tensor) and SPPF (three chained 5x5 stride-1 max-pools).
#pragma once
#include <cstdint>
#include "ixb_ptx.cuh"
#include "ixb_conv.cuh"

namespace ixb {

// uint8 pixels [B][3][H][W] -> int8 [B][H+2][W+4][8] (bytes 0..2 = lut[pixel] of the three channels,
// bytes 3..7 = 0; halo columns and rows are left untouched and stay zero). One thread per 4
// horizontally adjacent pixels. The lookup is the model input's QuantizeLinear
// (graph_session.py:144-149 input_lut).
__global__ void __launch_bounds__(256) quantize_images_kernel(const uint8_t* __restrict__ img,
                                                               const int8_t* __restrict__ lut, int B, int H,
                                                               int W, int8_t* __restrict__ out) {
  __shared__ uint8_t lut_s[256];
  grid_dep_launch();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut_s[i] = (uint8_t)lut[i];
  __syncthreads();
  grid_dep_wait();
  const int wq = W >> 2;
  const long long total = (long long)B * H * wq;
  const long long plane = (long long)H * W;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long b = i / ((long long)H * wq);
    const int rem = (int)(i - b * H * wq);
    const int y = rem / wq, x4 = (rem - (rem / wq) * wq) * 4;
    const uint8_t* src = img + b * 3 * plane + (long long)y * W + x4;
    const uint32_t r = __ldg(reinterpret_cast<const uint32_t*>(src));
    const uint32_t g = __ldg(reinterpret_cast<const uint32_t*>(src + plane));
    const uint32_t bl = __ldg(reinterpret_cast<const uint32_t*>(src + 2 * plane));
    uint2* dst = reinterpret_cast<uint2*>(out + ((b * (H + 2) + y + 1) * (long long)(W + 4) + x4 + 1) * 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w = (uint32_t)lut_s[(r >> (8 * j)) & 0xFF] | ((uint32_t)lut_s[(g >> (8 * j)) & 0xFF] << 8) |
                         ((uint32_t)lut_s[(bl >> (8 * j)) & 0xFF] << 16);
      dst[j] = make_uint2(w, 0u);
    }
  }
}

struct PoolParams {
  SegDev in;
  SegDev out[3];
  int H, W, chunks;
};

__device__ __forceinline__ uint4 vmax16(uint4 a, uint4 b) {
  return make_uint4(__vmaxs4(a.x, b.x), __vmaxs4(a.y, b.y), __vmaxs4(a.z, b.z), __vmaxs4(a.w, b.w));
}

// SPPF: out[k] = pool5^(k+1)(in) for k = 0, 1, 2, each a 5x5 stride-1 max with -128 padding
// (uint8 0 in the reference, graph_reference.py:64-72; three chained MaxPool layers,
// graph_ir.py:1120-1133). One CTA per (16-channel chunk plane, image); the image's plane lives
// in shared memory as 16-byte pixels and each pool is a row pass then a column pass of
// per-byte signed maxima. Out-of-image taps are skipped, which equals -128 padding because the
// window centre is always inside.
__global__ void __launch_bounds__(256) sppf_kernel(const __grid_constant__ PoolParams p) {
  extern __shared__ uint4 pool_smem[];
  const int n = p.H * p.W;
  uint4* cur = pool_smem;
  uint4* tmp = cur + n;
  uint4* nxt = tmp + n;
  const int chunk = blockIdx.x;
  const int img = blockIdx.y;
  const int W2 = p.W + 2;
  const int8_t* src = p.in.base + (long long)chunk * p.in.plane + (long long)img * p.in.P * 16;
  grid_dep_launch();
  grid_dep_wait();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int y = i / p.W, x = i - (i / p.W) * p.W;
    cur[i] = *reinterpret_cast<const uint4*>(src + ((y + 1) * W2 + x + 1) * 16);
  }
  __syncthreads();
  for (int k = 0; k < 3; ++k) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int y = i / p.W, x = i - (i / p.W) * p.W;
      uint4 m = cur[i];
      for (int d = -2; d <= 2; ++d)
        if (d != 0 && x + d >= 0 && x + d < p.W) m = vmax16(m, cur[y * p.W + x + d]);
      tmp[i] = m;
    }
    __syncthreads();
    int8_t* dst = const_cast<int8_t*>(p.out[k].base) + (long long)chunk * p.out[k].plane + (long long)img * p.out[k].P * 16;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int y = i / p.W, x = i - (i / p.W) * p.W;
      uint4 m = tmp[i];
      for (int d = -2; d <= 2; ++d)
        if (d != 0 && y + d >= 0 && y + d < p.H) m = vmax16(m, tmp[(y + d) * p.W + x]);
      nxt[i] = m;
      *reinterpret_cast<uint4*>(dst + ((y + 1) * W2 + x + 1) * 16) = m;
    }
    __syncthreads();
    uint4* t = cur;
    cur = nxt;
    nxt = t;
  }
}

}  // namespace ixb
