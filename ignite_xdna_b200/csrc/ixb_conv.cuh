// int8 implicit-GEMM convolution on the 5th-generation tensor cores (tcgen05, kind::i8),
// with the XINT8 epilogue fused: bias, pow2 shift-round-saturate, 256-entry activation table,
// residual add, and the store into the consumer's channel slice (or the NCHW head egress).
//
// Semantics: the conv of the reference's integer reference (graph_reference.py:40-61) in the
// int8 domain t = q - 128: acc = (bias_q << e) + sum w * t over a zero (t = 0) padded input,
// t1 = clamp(rne(acc >> shift), -128, 127), t2 = lut[t1], and with a residual
// y = clamp(rne((t2 << lsh_m) + (r << lsh_r), rsh), -128, 127) (engine_emulator.py:149-204).
// Because 128 << shift is a multiple of 2^shift, this equals the reference's uint8 rule
// sat_u8(rne(bias_acc + sum w * q)) - 128 exactly.
//
// GEMM view: M = output pixels (128 per CTA, one TMEM lane each), N = output channels
// (n_tile per CTA, one TMEM column each), K = input channels x taps in 32-byte steps.
// Activations are int8 NHWC with a one-pixel zero halo, so:
//  * WINDOW (stride 1, same resolution): the CTA computes 128 consecutive pixels of the
//    flattened padded image; tap (ky, kx) of output pixel m reads padded pixel
//    m + (ky-1)(W+2) + (kx-1), so ONE window of 128 + 2((W+2)+1) pixels per 32 input channels
//    feeds all nine taps: each tap is the same smem window seen through a descriptor whose
//    start address moves by 16 bytes per pixel of shift. Halo outputs are computed and dropped.
//  * GATHER (stride 2, or an input read through a nearest-2x upsample): the CTA computes 128
//    interior output pixels and gathers each tap's rows with 16-byte cp.async.
//  * STEM: the 3-channel image stored as 4-byte pixels; one 16-byte K-chunk is 4 pixels x
//    4 channels of one input row, so K = 3 rows x 16 bytes (+16 zero) covers the 3x3 window.
// Shared-memory operands use the K-major no-swizzle core-matrix layout: A as
// [chunk][pixel][16 B] (SBO 128 B, LBO = rows x 16 B), B as [n/8][chunk][8][16 B]
// (SBO 256 B, LBO 128 B), prepacked on the host so one bulk copy lands a K-block.
#pragma once
#include <cstdint>
#include "ixb_ptx.cuh"
#include "../../include/ixb200.h"

namespace ixb {

struct SegDev {
  const int8_t* base;    // padded pixel (0,0) of image 0
  long long img_stride;  // bytes per image
  int pitch, ch_off;
  int chunk_begin, chunks;  // 16-channel chunks of the logical input this view supplies
  int H, W, up2;
};

struct ConvParams {
  int mode, k, stride, pad;
  int H, W, Ho, Wo, batch;
  long long m_total;
  int cin_chunks, cp, kblocks, taps_per_block, pair_groups;
  int rowsA, win_origin;
  int a_stage_bytes, b_stage_bytes, stage_bytes, stages;
  int n_tile, tmem_cols;
  uint32_t idesc;
  int nseg;
  SegDev seg[IXB_MAX_SEGS];
  const uint8_t* wpack;
  long long w_ntile_stride;
  const int32_t* bias;
  const int8_t* lut;
  int shift;
  int has_res;
  SegDev res;
  int res_lsh_m, res_lsh_r, res_shift;
  int out_nchw;
  SegDev out;
  int8_t* egress;
  long long egress_img;
  int cout;
};

constexpr int kConvThreads = 128;
constexpr int kTileM = 128;

template <int MODE>
__device__ __forceinline__ void conv_load_a(const ConvParams& p, uint8_t* As, int kb, long long m0, int tid) {
  const int nch = 2 * p.cp;
  const int c = tid % nch;  // 128 is a multiple of nch, so each thread keeps one chunk
  const int step = kConvThreads / nch;
  uint8_t* dst = As + c * p.rowsA * 16;
  if (MODE == IXB_MODE_STEM) {
    const SegDev& s = p.seg[0];
    for (int r = tid / nch; r < kTileM; r += step) {
      const long long m = m0 + r;
      const bool ok = c < 3 && m < p.m_total;
      const int8_t* src = s.base;
      if (ok) {
        const long long hw = (long long)p.Ho * p.Wo;
        const long long img = m / hw;
        const int rem = (int)(m - img * hw);
        const int y = rem / p.Wo, x = rem - (rem / p.Wo) * p.Wo;
        // padded row 2y + ky, padded columns 2x .. 2x+3 (input columns 2x-1 .. 2x+2)
        src = s.base + img * s.img_stride + ((long long)(2 * y + c) * (s.W + 2) + 2 * x) * s.pitch;
      }
      cp_async8(dst + r * 16, src, ok ? 8u : 0u);
      cp_async8(dst + r * 16 + 8, ok ? src + 8 : src, ok ? 8u : 0u);
    }
    return;
  }
  int gc, tap = 0;
  if (MODE == IXB_MODE_WINDOW) {
    gc = kb * nch + c;
  } else {
    tap = kb / p.pair_groups;
    gc = (kb - tap * p.pair_groups) * nch + c;
  }
  int si = -1;
#pragma unroll
  for (int s = 0; s < IXB_MAX_SEGS; ++s)
    if (s < p.nseg && gc >= p.seg[s].chunk_begin && gc < p.seg[s].chunk_begin + p.seg[s].chunks) si = s;
  const bool cvalid = si >= 0;
  const SegDev& s = p.seg[cvalid ? si : 0];
  const int8_t* cbase = s.base + s.ch_off + (cvalid ? (gc - s.chunk_begin) * 16 : 0);
  if (MODE == IXB_MODE_WINDOW) {
    const long long wb = m0 - p.win_origin;
    for (int px = tid / nch; px < p.rowsA; px += step) {
      const long long m = wb + px;
      const bool ok = cvalid && m >= 0 && m < p.m_total;
      cp_async16(dst + px * 16, ok ? cbase + m * s.pitch : s.base, ok ? 16u : 0u);
    }
  } else {
    const int ky = tap / p.k, kx = tap - (tap / p.k) * p.k;
    const long long hw = (long long)p.Ho * p.Wo;
    for (int r = tid / nch; r < kTileM; r += step) {
      const long long m = m0 + r;
      const bool ok = cvalid && m < p.m_total;
      const int8_t* src = s.base;
      if (ok) {
        const long long img = m / hw;
        const int rem = (int)(m - img * hw);
        const int y = rem / p.Wo, x = rem - (rem / p.Wo) * p.Wo;
        int iy = y * p.stride + ky - p.pad, ix = x * p.stride + kx - p.pad;
        if (s.up2) { iy >>= 1; ix >>= 1; }
        src = cbase + img * s.img_stride + ((long long)(iy + 1) * (s.W + 2) + (ix + 1)) * s.pitch;
      }
      cp_async16(dst + r * 16, src, ok ? 16u : 0u);
    }
  }
}

template <int MODE, int S>
__global__ void __launch_bounds__(kConvThreads) conv_kernel(const __grid_constant__ ConvParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint64_t* bfull = reinterpret_cast<uint64_t*>(smem + S * p.stage_bytes);
  uint64_t* mdone = bfull + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + S);
  int8_t* lut_s = reinterpret_cast<int8_t*>(smem + S * p.stage_bytes + 256);

  const long long m0 = (long long)blockIdx.x * kTileM;
  const int ntile = blockIdx.y;
  const int KB = p.kblocks;

  if (warp == 0) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&mdone[s], 1);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < 256; i += kConvThreads) lut_s[i] = p.lut[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto load_stage = [&](int kb) {
    const int st = kb % S;
    uint8_t* As = smem + st * p.stage_bytes;
    uint8_t* Bs = As + p.a_stage_bytes;
    conv_load_a<MODE>(p, As, kb, m0, tid);
    if (tid == 0) {
      mbar_arrive_expect_tx(&bfull[st], p.b_stage_bytes);
      bulk_g2s(Bs, p.wpack + ntile * p.w_ntile_stride + (long long)kb * p.b_stage_bytes, p.b_stage_bytes,
               &bfull[st]);
    }
  };

  // L K-blocks of loads run ahead of the MMAs; S - L K-blocks of MMAs may be in flight.
  constexpr int L = (S >= 4) ? S - 2 : S - 1;
#pragma unroll
  for (int s = 0; s < L; ++s) {
    if (s < KB) load_stage(s);
    cp_async_commit();
  }

  for (int kb = 0; kb < KB; ++kb) {
    const int st = kb % S;
    const int nk = kb + L;
    if (nk < KB) {
      const int prev = nk - S;  // the K-block that last used stage nk % S
      if (prev >= 0) mbar_wait(&mdone[prev % S], (prev / S) & 1);
      load_stage(nk);
    }
    cp_async_commit();
    cp_async_wait<L>();
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      mbar_wait(&bfull[st], (kb / S) & 1);
      tc_fence_after();
      const uint32_t a0 = smem_u32(smem + st * p.stage_bytes);
      const uint32_t b0 = a0 + p.a_stage_bytes;
      const uint32_t lbo_a = p.rowsA * 16;
      int i = 0;
      for (int pp = 0; pp < p.cp; ++pp) {
        for (int t = 0; t < p.taps_per_block; ++t) {
          uint32_t shift_px = 0;
          if (MODE == IXB_MODE_WINDOW) shift_px = (t / p.k) * (p.W + 2) + (t - (t / p.k) * p.k);
          const uint64_t ad = umma_desc(a0 + pp * 2 * lbo_a + shift_px * 16, lbo_a, 128);
          const uint64_t bd = umma_desc(b0 + (pp * p.taps_per_block + t) * p.n_tile * 32, 128, 256);
          umma_s8(tmem, ad, bd, p.idesc, (kb > 0 || i > 0) ? 1u : 0u);
          ++i;
        }
      }
      umma_commit(&mdone[st]);
    }
  }
  if (KB > 0) mbar_wait(&mdone[(KB - 1) % S], ((KB - 1) / S) & 1);
  tc_fence_after();

  // ---------------------------------------------------------------- epilogue
  const int row = warp * 32 + lane;
  const long long m = m0 + row;
  bool valid = m < p.m_total;
  long long opix = 0;
  long long img = 0;
  int oy = 0, ox = 0;
  if (MODE == IXB_MODE_WINDOW) {
    const long long P = (long long)(p.H + 2) * (p.W + 2);
    img = m / P;
    const int rem = (int)(m - img * P);
    const int yp = rem / (p.W + 2), xp = rem - (rem / (p.W + 2)) * (p.W + 2);
    valid = valid && yp >= 1 && yp <= p.H && xp >= 1 && xp <= p.W;
    opix = m;
    oy = yp - 1;
    ox = xp - 1;
  } else {
    const long long hw = (long long)p.Ho * p.Wo;
    img = m / hw;
    const int rem = (int)(m - img * hw);
    oy = rem / p.Wo;
    ox = rem - oy * p.Wo;
    opix = img * (long long)(p.Ho + 2) * (p.Wo + 2) + (long long)(oy + 1) * (p.Wo + 2) + (ox + 1);
  }
  const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
  for (int j = 0; j < p.n_tile / 16; ++j) {
    uint32_t v[16];
    tmem_ld16(tl + j * 16, v);
    tmem_ld_wait();
    if (!valid) continue;
    const int co = ntile * p.n_tile + j * 16;
    int bias[16];
    {
      const int4* bp = reinterpret_cast<const int4*>(p.bias + co);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int4 b4 = __ldg(bp + q);
        bias[4 * q] = b4.x; bias[4 * q + 1] = b4.y; bias[4 * q + 2] = b4.z; bias[4 * q + 3] = b4.w;
      }
    }
    int8_t rv[16];
    if (p.has_res) {
      const uint4 r4 = *reinterpret_cast<const uint4*>(p.res.base + opix * p.res.pitch + p.res.ch_off + co);
      *reinterpret_cast<uint4*>(rv) = r4;
    }
    alignas(16) int8_t ov[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int a = (int)v[i] + bias[i];
      int t = lut_s[clamp_i8(rne_shift(a, p.shift)) + 128];
      if (p.has_res)
        t = clamp_i8(rne_shift((t << p.res_lsh_m) + ((int)rv[i] << p.res_lsh_r), p.res_shift));
      ov[i] = (int8_t)t;
    }
    if (!p.out_nchw) {
      *reinterpret_cast<uint4*>(const_cast<int8_t*>(p.out.base) + opix * p.out.pitch + p.out.ch_off + co) =
          *reinterpret_cast<const uint4*>(ov);
    } else {
      int8_t* e = p.egress + img * p.egress_img + (long long)oy * p.Wo + ox;
      const long long plane = (long long)p.Ho * p.Wo;
#pragma unroll
      for (int i = 0; i < 16; ++i) e[(co + i) * plane] = ov[i];
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, p.tmem_cols);
}

}  // namespace ixb
