// Bandwidth-bound kernels of the XINT8 graph: image ingress (pixel -> int8 lookup into the
// padded 8-byte-pixel stem tensor) and SPPF (three chained 5x5 stride-1 max-pools).
#pragma once
#include <cstdint>
#include "ixb_ptx.cuh"
#include "ixb_conv.cuh"

namespace ixb {

// uint8 pixels [B][3][H][W] -> int8 [B][H+2][W+4][8] (bytes 0..2 = lut[pixel] of the three channels,
// bytes 3..7 = 0). One thread per 16-byte pixel pair of the padded row: pair k covers padded
// columns 2k and 2k + 1, i.e. image columns 2k - 1 and 2k (column -1 and column W are the zero
// halo, written as zeros), so a warp's stores are 512 contiguous bytes of whole sectors. Halo rows
// and padded columns past W + 1 are left untouched and stay zero. The item index splits into
// (image, row, pair) by multiply-shift divisions (items < 2^31). The lookup is the model input's
// QuantizeLinear (graph_session.py:144-149 input_lut).
__global__ void __launch_bounds__(256) quantize_images_kernel(const uint8_t* __restrict__ img,
                                                               const int8_t* __restrict__ lut, int B, int H,
                                                               int W, FastDiv fd_pairs, FastDiv fd_h,
                                                               int8_t* __restrict__ out) {
  __shared__ uint8_t lut_s[256];
  grid_dep_launch();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut_s[i] = (uint8_t)lut[i];
  __syncthreads();
  grid_dep_wait();
  const int pairs = W / 2 + 1;
  const int total = B * H * pairs;
  const long long plane = (long long)H * W;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int row = (int)fdiv((uint32_t)i, fd_pairs);  // b * H + y
    const int k = i - row * pairs;
    const int b = (int)fdiv((uint32_t)row, fd_h), y = row - b * H;
    const uint8_t* src = img + (long long)b * 3 * plane + (long long)y * W;
    auto px = [&](int x) -> uint32_t {
      if (x < 0 || x >= W) return 0u;
      return (uint32_t)lut_s[__ldg(src + x)] | ((uint32_t)lut_s[__ldg(src + plane + x)] << 8) |
             ((uint32_t)lut_s[__ldg(src + 2 * plane + x)] << 16);
    };
    const uint32_t w0 = px(2 * k - 1), w1 = px(2 * k);
    *reinterpret_cast<uint4*>(out + (((long long)b * (H + 2) + y + 1) * (W + 4) + 2 * k) * 8) = make_uint4(w0, 0u, w1, 0u);
  }
}

// Letterbox ingress: a BGR uint8 frame (any size, row stride) -> letterboxed, Q11-bilinear
// resized, quantized 8-byte pixels (bytes 0..2 = lut[R], lut[G], lut[B]) in the stem's padded input,
// the same bytes as the reference's pipelines/preprocess_simd.c fused_preprocess_bgr_to_c8_plane
// (:331-590): scale = min(dst / src) in float32, nw/nh = floor(src * scale + 0.5), centred pads,
// per output column sx = (x + 0.5) * (src_w / nw) - 0.5 clamped at the edges with the weight
// bx1 = floor(alpha * 2048 + 0.5) (float32, written with round-to-nearest intrinsics so nothing
// contracts), rows likewise, then ((p00 bx0 + p01 bx1 + 1024) >> 11) by0 + (...) by1 + 1024 >> 11
// in integers; outside the resized image the pad pixel lut[114]. One thread per output pixel.
struct LetterboxParams {
  const uint8_t* frames;
  long long frame_bytes;
  int src_w, src_h, src_stride;
  int dst_w, dst_h, nw, nh, pad_top, pad_left;
  float fx, fy;
  const int8_t* lut;
  int8_t* out;           // pixel (0, 0) of image 0 in the padded input
  int out_row_pixels;    // padded row length in 8-byte pixels
  long long out_image_bytes;
  int batch;
};

__device__ __forceinline__ void letterbox_axis(int i, float f, int src, int& i0, int& i1, int& w0, int& w1) {
  const float sv = __fsub_rn(__fmul_rn(__fadd_rn((float)i, 0.5f), f), 0.5f);
  int a = (int)floorf(sv);
  if (a < 0) a = 0;
  int b = a + 1;
  if (b >= src) b = src - 1;
  float al = __fsub_rn(sv, (float)a);
  al = fminf(fmaxf(al, 0.0f), 1.0f);
  const int wb = (int)floorf(__fadd_rn(__fmul_rn(al, 2048.0f), 0.5f));
  i0 = a;
  i1 = b;
  w0 = 2048 - wb;
  w1 = wb;
}

__global__ void __launch_bounds__(256) letterbox_kernel(const __grid_constant__ LetterboxParams p) {
  __shared__ int8_t lut_s[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut_s[i] = p.lut[i];
  __syncthreads();
  const long long total = (long long)p.batch * p.dst_h * p.dst_w;
  const uint32_t pad = (uint8_t)lut_s[114] * 0x010101u;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (long long)gridDim.x * blockDim.x) {
    const int img = (int)(t / ((long long)p.dst_h * p.dst_w));
    const int rem = (int)(t - (long long)img * p.dst_h * p.dst_w);
    const int y = rem / p.dst_w, x = rem - y * p.dst_w;
    const int iy = y - p.pad_top, ix = x - p.pad_left;
    uint32_t v = pad;
    if (iy >= 0 && iy < p.nh && ix >= 0 && ix < p.nw) {
      int x0, x1, bx0, bx1, y0, y1, by0, by1;
      letterbox_axis(ix, p.fx, p.src_w, x0, x1, bx0, bx1);
      letterbox_axis(iy, p.fy, p.src_h, y0, y1, by0, by1);
      const uint8_t* f = p.frames + (long long)img * p.frame_bytes;
      const uint8_t* r0 = f + (long long)y0 * p.src_stride;
      const uint8_t* r1 = f + (long long)y1 * p.src_stride;
      uint32_t o = 0;
#pragma unroll
      for (int c = 0; c < 3; ++c) {  // source B, G, R -> output bytes 2, 1, 0
        const int top = (r0[x0 * 3 + c] * bx0 + r0[x1 * 3 + c] * bx1 + 1024) >> 11;
        const int bot = (r1[x0 * 3 + c] * bx0 + r1[x1 * 3 + c] * bx1 + 1024) >> 11;
        const int val = (top * by0 + bot * by1 + 1024) >> 11;
        o |= (uint32_t)(uint8_t)lut_s[val] << (8 * (2 - c));
      }
      v = o;
    }
    *reinterpret_cast<uint2*>(p.out + img * p.out_image_bytes + ((long long)y * p.out_row_pixels + x) * 8) =
        make_uint2(v, 0u);
  }
}

// Image ingress into its space-to-depth view (the stem's input when the stem runs as a 2x2
// WINDOW conv): uint8 pixels [B][3][H][W] -> 16-byte pixels of the (H/2) x (W/2) view, byte
// ph * 3 + c = lut[channel c of image pixel (2 sy + ry, 2 sx + rx)], ph = 2 ry + rx, bytes 12..15
// zero. One thread per two neighbouring view pixels: four-pixel (4-byte) loads from each channel's
// two rows (W % 4 == 0). The lookup is the model input's QuantizeLinear (graph_session.py:144-149
// input_lut). `out` is padded pixel 0 of image 0; P2 / W2 are the view's padded pixels per image
// and padded width; fd_w divides by W / 4.
__global__ void __launch_bounds__(256) quantize_images_s2d_kernel(const uint8_t* __restrict__ img,
                                                                   const int8_t* __restrict__ lut, int B, int H,
                                                                   int W, FastDiv fd_w, FastDiv fd_h, int P2, int W2,
                                                                   int8_t* __restrict__ out) {
  __shared__ uint8_t lut_s[256];
  grid_dep_launch();
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut_s[i] = (uint8_t)lut[i];
  __syncthreads();
  grid_dep_wait();
  const int hq = W / 4, hh = H / 2;  // view pixel pairs per row, view rows
  const int total = B * hh * hq;
  const long long plane = (long long)H * W;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int row = (int)fdiv((uint32_t)i, fd_w);  // b * hh + sy
    const int k = i - row * hq;                     // view pixels 2k, 2k + 1
    const int b = (int)fdiv((uint32_t)row, fd_h), sy = row - b * hh;
    const uint8_t* src = img + (long long)b * 3 * plane + (long long)(2 * sy) * W + 4 * k;
    uint32_t q[2][12];  // q[view pixel][ph * 3 + c]
#pragma unroll
    for (int c = 0; c < 3; ++c) {
#pragma unroll
      for (int ry = 0; ry < 2; ++ry) {
        const uint32_t four = __ldg(reinterpret_cast<const uint32_t*>(src + c * plane + ry * W));
#pragma unroll
        for (int j = 0; j < 4; ++j)  // image column 4k + j: view pixel j / 2, phase column j % 2
          q[j >> 1][(2 * ry + (j & 1)) * 3 + c] = lut_s[(four >> (8 * j)) & 0xFF];
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + ((long long)b * P2 + (long long)(sy + 1) * W2 + 2 * k + 1) * 16);
#pragma unroll
    for (int v = 0; v < 2; ++v)
      dst[v] = make_uint4(q[v][0] | (q[v][1] << 8) | (q[v][2] << 16) | (q[v][3] << 24),
                          q[v][4] | (q[v][5] << 8) | (q[v][6] << 16) | (q[v][7] << 24),
                          q[v][8] | (q[v][9] << 8) | (q[v][10] << 16) | (q[v][11] << 24), 0u);
  }
}

// The 8-byte-pixel image store [B][H+2][W+4][8] (pixel (y, x) at padded (y + 1, x + 1)) ->
// the space-to-depth view above: after ixb_session_letterbox, which writes the 8-byte layout.
__global__ void __launch_bounds__(256) repack_s2d_kernel(const int8_t* __restrict__ in, int B, int H, int W,
                                                          FastDiv fd_w, FastDiv fd_h, int P2, int W2,
                                                          int8_t* __restrict__ out) {
  const int hw = W / 2, hh = H / 2;
  const int total = B * hh * hw;
  const int R = W + 4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int row = (int)fdiv((uint32_t)i, fd_w);
    const int sx = i - row * hw;
    const int b = (int)fdiv((uint32_t)row, fd_h), sy = row - b * hh;
    uint32_t q[12];
#pragma unroll
    for (int ph = 0; ph < 4; ++ph) {
      const int y = 2 * sy + (ph >> 1), x = 2 * sx + (ph & 1);
      const uint32_t px = *reinterpret_cast<const uint32_t*>(in + (((long long)b * (H + 2) + y + 1) * R + x + 1) * 8);
      q[ph * 3] = px & 0xFF;
      q[ph * 3 + 1] = (px >> 8) & 0xFF;
      q[ph * 3 + 2] = (px >> 16) & 0xFF;
    }
    const uint32_t w0 = q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24);
    const uint32_t w1 = q[4] | (q[5] << 8) | (q[6] << 16) | (q[7] << 24);
    const uint32_t w2 = q[8] | (q[9] << 8) | (q[10] << 16) | (q[11] << 24);
    *reinterpret_cast<uint4*>(out + ((long long)b * P2 + (long long)(sy + 1) * W2 + sx + 1) * 16) =
        make_uint4(w0, w1, w2, 0u);
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

// SPPF for planes of at most 1024 pixels (YOLOv8's 20x20 at 640): the same three pools, one
// thread per pixel (blockDim = n rounded up to whole warps), so each thread splits its pixel index
// once instead of dividing for every pixel of every pass.
__global__ void __launch_bounds__(1024) sppf_pixel_kernel(const __grid_constant__ PoolParams p) {
  extern __shared__ uint4 pool_px[];
  const int W = p.W, H = p.H, n = H * W;
  uint4* cur = pool_px;
  uint4* tmp = cur + n;
  uint4* nxt = tmp + n;
  const int t = threadIdx.x;
  const bool on = t < n;
  const int y = on ? t / W : 0, x = on ? t - (t / W) * W : 0;
  const int chunk = blockIdx.x, img = blockIdx.y;
  const int W2 = W + 2;
  const int8_t* src = p.in.base + (long long)chunk * p.in.plane + (long long)img * p.in.P * 16;
  grid_dep_launch();
  grid_dep_wait();
  if (on) cur[t] = *reinterpret_cast<const uint4*>(src + ((y + 1) * W2 + x + 1) * 16);
  __syncthreads();
  for (int k = 0; k < 3; ++k) {
    if (on) {
      uint4 m = cur[t];
      if (x >= 1) m = vmax16(m, cur[t - 1]);
      if (x >= 2) m = vmax16(m, cur[t - 2]);
      if (x + 1 < W) m = vmax16(m, cur[t + 1]);
      if (x + 2 < W) m = vmax16(m, cur[t + 2]);
      tmp[t] = m;
    }
    __syncthreads();
    if (on) {
      uint4 m = tmp[t];
      if (y >= 1) m = vmax16(m, tmp[t - W]);
      if (y >= 2) m = vmax16(m, tmp[t - 2 * W]);
      if (y + 1 < H) m = vmax16(m, tmp[t + W]);
      if (y + 2 < H) m = vmax16(m, tmp[t + 2 * W]);
      nxt[t] = m;
      int8_t* dst = const_cast<int8_t*>(p.out[k].base) + (long long)chunk * p.out[k].plane + (long long)img * p.out[k].P * 16;
      *reinterpret_cast<uint4*>(dst + ((y + 1) * W2 + x + 1) * 16) = m;
    }
    __syncthreads();
    uint4* s = cur;
    cur = nxt;
    nxt = s;
  }
}

// Self-check of the bounded waits: one thread waits on an mbarrier that nothing arrives at, with a
// limit of limit_ns; the wait gives up, raises DEV_ERR_WAIT_TIMEOUT in the device flag and the
// kernel returns normally (no trap, no fault: the context stays usable).
__global__ void bounded_wait_probe_kernel(unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_for(&bar, 0, limit_ns);
}

}  // namespace ixb
