// YOLOv8 detect-head decode on the GPU: the per-anchor int8 confidence prune on the class
// maximum, the class score from the sigmoid table, the DFL expectation over 16 bins, box
// reconstruction with letterbox removal, then class-batched greedy NMS -- the detections of the
// reference's pipelines/decode_native.c (yolo_decode_int8, :407-540), bit for bit:
//   * float32 operations in the reference's order (the 16 bins accumulate in index order; the
//     division and products are IEEE round-to-nearest, written as __f*_rn so nothing contracts
//     into an FMA); every exp comes from the caller's tables (dfl_exp, sigmoid), built on the host
//     with numpy exactly as the reference builds them;
//   * the class is the first whose logit reaches sigmoid_low[q_max] (numpy's argmax over float32
//     probabilities), or a plain first-maximum argmax over the sigmoid values without that table;
//   * NMS as OpenCV's NMSBoxesBatched: boxes offset by class * (max coordinate + 1) in double,
//     scores strictly above the threshold stably sorted in descending order, a box kept when its
//     overlap 1 - (float)(1 - inter / union) with every kept box is at most the IoU threshold.
// One CTA decodes one image; its candidates live in shared memory (no scratch in global memory).
#pragma once
#include <cfloat>
#include <cstdint>
#include "../../include/ixb200.h"

namespace ixb {

constexpr int kDecodeThreads = 1024;
constexpr int kDecodeMaxAnchors = 8400;
constexpr int kDfl = 16;

struct DecodeHeadDev {
  long long box_off, cls_off;   // byte offsets of the box and class heads inside one image's egress
  const float* dfl_exp;         // [256][256]
  const float* sigmoid;         // [256]
  const int32_t* sigmoid_low;   // [256] or null
  int qi;                       // integer prune threshold: an anchor survives when its class max > qi
  int anchors, anchor_offset;
};

struct DecodeParams {
  const int8_t* egress;
  long long egress_image_bytes;
  DecodeHeadDev head[3];
  const float* anchor_x;
  const float* anchor_y;
  const float* strides;
  int num_classes;
  float conf, iou;
  const float* letterbox;       // [B][3]: pad_top, pad_left, scale
  int capacity;
  float* out_box;               // [B][capacity][4]: x0, y0, w, h
  float* out_score;             // [B][capacity]
  int32_t* out_class;           // [B][capacity]
  int32_t* out_count;           // [B]: detections, or -3 when more than `capacity` survive NMS
};

__device__ __forceinline__ float dfl_side(const int8_t* box, int n, int a, int side, const float* dfl_exp) {
  int q[kDfl];
  int q_max = -128;
#pragma unroll
  for (int k = 0; k < kDfl; ++k) {
    q[k] = box[(long long)(side * kDfl + k) * n + a];
    q_max = max(q_max, q[k]);
  }
  const float* row = dfl_exp + (q_max + 128) * 256;
  float e[kDfl];
#pragma unroll
  for (int k = 0; k < kDfl; ++k) e[k] = __ldg(row + q[k] + 128);
  float sum = e[0];
#pragma unroll
  for (int k = 1; k < kDfl; ++k) sum = __fadd_rn(sum, e[k]);
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < kDfl; ++k) {
    const float w = __fmul_rn(__fdiv_rn(e[k], sum), (float)k);
    acc = k == 0 ? w : __fadd_rn(acc, w);
  }
  return acc;
}

// Area of the intersection of two class-offset boxes, as OpenCV's Rect2d operator& computes it.
__device__ __forceinline__ double inter_area(double ax, double ay, double aw, double ah, double bx, double by,
                                             double bw, double bh) {
  if (aw <= 0 || ah <= 0 || bw <= 0 || bh <= 0) return 0.0;
  const bool a_left = ax < bx, a_top = ay < by;
  const double xmin_x = a_left ? ax : bx, xmin_w = a_left ? aw : bw, xmax_x = a_left ? bx : ax, xmax_w = a_left ? bw : aw;
  const double ymin_y = a_top ? ay : by, ymin_h = a_top ? ah : bh, ymax_y = a_top ? by : ay, ymax_h = a_top ? bh : ah;
  if ((xmin_x < 0 && __dadd_rn(xmin_x, xmin_w) < xmax_x) || (ymin_y < 0 && __dadd_rn(ymin_y, ymin_h) < ymax_y))
    return 0.0;
  const double wx = __dsub_rn(xmin_w, __dsub_rn(xmax_x, xmin_x));
  const double w = (xmax_w < wx) ? xmax_w : wx;
  const double hy = __dsub_rn(ymin_h, __dsub_rn(ymax_y, ymin_y));
  const double h = (ymax_h < hy) ? ymax_h : hy;
  if (w <= 0 || h <= 0) return 0.0;
  return __dmul_rn(w, h);
}

// The suppression test of the greedy NMS: overlap 1 - (float)(1 - inter / union) of two
// class-offset boxes, > iou (or unordered: NaN) suppresses; boxes whose areas add up to at most
// DBL_EPSILON count as overlap 1 (OpenCV's rule).
__device__ __forceinline__ bool suppresses(float4 bi, double oi, float4 bk, double ok, float iou) {
  const double ix = __dadd_rn((double)bi.x, oi), iy = __dadd_rn((double)bi.y, oi);
  const double iw = bi.z, ih = bi.w, iarea = __dmul_rn(iw, ih);
  const double kx = __dadd_rn((double)bk.x, ok), ky = __dadd_rn((double)bk.y, ok);
  const double kw = bk.z, kh = bk.w, karea = __dmul_rn(kw, kh);
  float ov;
  if (__dadd_rn(iarea, karea) <= DBL_EPSILON) {
    ov = 1.0f;
  } else {
    const double inter = inter_area(ix, iy, iw, ih, kx, ky, kw, kh);
    const double uni = __dsub_rn(__dadd_rn(iarea, karea), inter);
    // Most pairs are decided without the division: inter <= union, so inter - iou * union is
    // computed to ~1e-16 * union, and a margin of 1e-6 * union puts inter / union on one side of
    // iou by far more than the double division and the float conversions round (~1e-7).
    if (iou >= 0.f && iou <= 1.f) {
      const double dlt = __dsub_rn(inter, __dmul_rn((double)iou, uni)), margin = __dmul_rn(1e-6, uni);
      if (dlt > margin) return true;
      if (dlt < -margin) return false;
    }
    ov = __fsub_rn(1.0f, __double2float_rn(__dsub_rn(1.0, __ddiv_rn(inter, uni))));
  }
  return !(ov <= iou);
}

__global__ void __launch_bounds__(kDecodeThreads, 1) yolo_decode_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ uint8_t dsmem[];
  float* s_score = reinterpret_cast<float*>(dsmem);                       // [8400]
  float4* s_box = reinterpret_cast<float4*>(s_score + kDecodeMaxAnchors);  // [8400] x0, y0, w, h
  int16_t* s_anchor = reinterpret_cast<int16_t*>(s_box + kDecodeMaxAnchors);  // [8400] anchor index
  uint8_t* s_class = reinterpret_cast<uint8_t*>(s_anchor + kDecodeMaxAnchors);  // [8400]
  uint16_t* s_order = reinterpret_cast<uint16_t*>(s_class + kDecodeMaxAnchors); // [16384] sort / kept list
  __shared__ int s_n, s_kept, s_nv;
  __shared__ double s_maxc[kDecodeThreads / 32];
  __shared__ uint16_t s_chunk[32];
  __shared__ unsigned s_mask[32];
  __shared__ int s_sup[32];

  const int img = blockIdx.x, tid = threadIdx.x;
  const int8_t* eg = p.egress + (long long)img * p.egress_image_bytes;
  const float pad_top = p.letterbox[3 * img], pad_left = p.letterbox[3 * img + 1], lscale = p.letterbox[3 * img + 2];
  if (tid == 0) {
    s_n = 0;
    s_kept = 0;
  }
  __syncthreads();

  // 1. candidates: prune, class score, DFL, box (shared-memory slots in any order; the sort below
  //    orders them by score and anchor, which is the reference's order after its stable sort)
  for (int h = 0; h < 3; ++h) {
    const DecodeHeadDev& hd = p.head[h];
    const int n = hd.anchors;
    const int8_t* box = eg + hd.box_off;
    const int8_t* cls = eg + hd.cls_off;
    for (int a = tid; a < n; a += kDecodeThreads) {
      int q_max = -128;
      for (int c = 0; c < p.num_classes; ++c) q_max = max(q_max, (int)cls[(long long)c * n + a]);
      if (q_max <= hd.qi) continue;
      float best;
      int best_c = 0;
      if (hd.sigmoid_low) {
        best = __ldg(hd.sigmoid + q_max + 128);
        if (!(best >= p.conf)) continue;
        const int lo = __ldg(hd.sigmoid_low + q_max + 128);
        while (best_c < p.num_classes - 1 && (int)cls[(long long)best_c * n + a] < lo) ++best_c;
      } else {
        best = __ldg(hd.sigmoid + (int)cls[a] + 128);
        for (int c = 1; c < p.num_classes; ++c) {
          const float pr = __ldg(hd.sigmoid + (int)cls[(long long)c * n + a] + 128);
          if (pr > best) {
            best = pr;
            best_c = c;
          }
        }
        if (!(best >= p.conf)) continue;
      }
      const float l = dfl_side(box, n, a, 0, hd.dfl_exp);
      const float t = dfl_side(box, n, a, 1, hd.dfl_exp);
      const float r = dfl_side(box, n, a, 2, hd.dfl_exp);
      const float b = dfl_side(box, n, a, 3, hd.dfl_exp);
      const int ai = hd.anchor_offset + a;
      const float ax = __ldg(p.anchor_x + ai), ay = __ldg(p.anchor_y + ai), st = __ldg(p.strides + ai);
      const float x1 = __fsub_rn(ax, l), y1 = __fsub_rn(ay, t), x2 = __fadd_rn(ax, r), y2 = __fadd_rn(ay, b);
      const float cx = __fmul_rn(__fmul_rn(__fadd_rn(x1, x2), 0.5f), st);
      const float cy = __fmul_rn(__fmul_rn(__fadd_rn(y1, y2), 0.5f), st);
      const float bw = __fmul_rn(__fsub_rn(x2, x1), st);
      const float bh = __fmul_rn(__fsub_rn(y2, y1), st);
      const int slot = atomicAdd(&s_n, 1);
      s_score[slot] = best;
      s_box[slot] = make_float4(__fdiv_rn(__fsub_rn(__fsub_rn(cx, __fdiv_rn(bw, 2.0f)), pad_left), lscale),
                                __fdiv_rn(__fsub_rn(__fsub_rn(cy, __fdiv_rn(bh, 2.0f)), pad_top), lscale),
                                __fdiv_rn(bw, lscale), __fdiv_rn(bh, lscale));
      s_anchor[slot] = (int16_t)ai;
      s_class[slot] = (uint8_t)best_c;
    }
  }
  __syncthreads();
  const int n = s_n;
  if (n == 0) {
    if (tid == 0) p.out_count[img] = 0;
    return;
  }

  // 2. the class offset of NMSBoxesBatched: max over every candidate's corners, starting at 0
  double mc = 0.0;
  for (int i = tid; i < n; i += kDecodeThreads) {
    const float4 bx = s_box[i];
    const double x1 = bx.x, y1 = bx.y, x2 = __dadd_rn(x1, (double)bx.z), y2 = __dadd_rn(y1, (double)bx.w);
    mc = fmax(mc, fmax(fmax(x1, y1), fmax(x2, y2)));
  }
  for (int o = 16; o > 0; o >>= 1) mc = fmax(mc, __shfl_xor_sync(0xffffffffu, mc, o));
  if ((tid & 31) == 0) s_maxc[tid >> 5] = mc;

  // 3. order: score descending, then anchor ascending (bitonic sort of slot ids, padded to 2^k)
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  for (int i = tid; i < np2; i += kDecodeThreads) s_order[i] = (uint16_t)(i < n ? i : 0xFFFF);
  __syncthreads();
  auto before = [&](uint16_t x, uint16_t y) -> bool {  // x strictly precedes y
    if (y == 0xFFFF) return x != 0xFFFF;
    if (x == 0xFFFF) return false;
    const float sx = s_score[x], sy = s_score[y];
    return sx > sy || (sx == sy && s_anchor[x] < s_anchor[y]);
  };
  for (int k = 2; k <= np2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += kDecodeThreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint16_t x = s_order[i], y = s_order[ixj];
          const bool up = (i & k) == 0;
          if (up ? before(y, x) : before(x, y)) {
            s_order[i] = y;
            s_order[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  double maxc = 0.0;
  for (int w = 0; w < kDecodeThreads / 32; ++w) maxc = fmax(maxc, s_maxc[w]);
  const double off_step = __dadd_rn(maxc, 1.0);

  // 4. Greedy NMS over the global order, 32 candidates at a time. A candidate is kept when no
  //    earlier kept candidate suppresses it. For a chunk of 32 (in order): every warp takes one
  //    candidate and its lanes test it against all candidates kept before the chunk; then the
  //    chunk's own 32 x 32 pairs are tested (thread (a, b): does earlier b suppress later a);
  //    then one warp resolves the chunk in order (a candidate survives if nothing kept before the
  //    chunk and no kept earlier member of the chunk suppresses it) and appends the kept ones.
  //    Exactly the sequential greedy loop, with a block barrier per 32 candidates instead of per
  //    candidate. Kept ids overwrite the front of s_order, behind the chunk being read.
  if (tid == 0) s_nv = n;
  __syncthreads();
  for (int i = tid; i < n; i += kDecodeThreads)
    if (!(s_score[s_order[i]] > p.conf)) atomicMin(&s_nv, i);  // the rest: a prefix of the order
  __syncthreads();
  const int nv = s_nv;
  const int warp = tid >> 5, lane = tid & 31;
  for (int r0 = 0; r0 < nv; r0 += 32) {
    const int cn = min(32, nv - r0);
    if (tid < 32) s_chunk[tid] = tid < cn ? s_order[r0 + tid] : (uint16_t)0;
    __syncthreads();
    const int kept = s_kept;
    if (warp < cn) {
      const uint16_t ci = s_chunk[warp];
      const float4 bi = s_box[ci];
      const double oi = __dmul_rn((double)s_class[ci], off_step);
      // kept candidates 32 at a time, stopping at the first group that suppresses this one (most
      // suppressed candidates meet their suppressor among the first, highest-scoring kept boxes)
      bool by_kept = false;
      for (int k0 = 0; k0 < kept && !by_kept; k0 += 32) {
        const int k = k0 + lane;
        bool sup = false;
        if (k < kept) {
          const uint16_t ck = s_order[k];
          sup = suppresses(bi, oi, s_box[ck], __dmul_rn((double)s_class[ck], off_step), p.iou);
        }
        by_kept = __any_sync(0xffffffffu, sup);
      }
      // earlier chunk members b < warp that would suppress this one if kept
      bool m = false;
      if (lane < warp) {
        const uint16_t cb = s_chunk[lane];
        m = suppresses(bi, oi, s_box[cb], __dmul_rn((double)s_class[cb], off_step), p.iou);
      }
      const unsigned mask = __ballot_sync(0xffffffffu, m);
      if (lane == 0) {
        s_mask[warp] = mask;
        s_sup[warp] = by_kept ? 1 : 0;
      }
    }
    __syncthreads();
    if (warp == 0) {
      // in order: a survives unless suppressed by an earlier kept candidate
      unsigned keep = 0u;
      for (int a = 0; a < cn; ++a)
        if (!s_sup[a] && !(s_mask[a] & keep)) keep |= 1u << a;
      if ((keep >> lane) & 1u) s_order[kept + __popc(keep & ((1u << lane) - 1u))] = s_chunk[lane];
      if (lane == 0) s_kept = kept + __popc(keep);
    }
    __syncthreads();
  }

  // 5. detections in kept order
  const int kept = s_kept;
  if (kept > p.capacity) {
    if (tid == 0) p.out_count[img] = -3;
    return;
  }
  for (int k = tid; k < kept; k += kDecodeThreads) {
    const uint16_t c = s_order[k];
    const long long o = (long long)img * p.capacity + k;
    reinterpret_cast<float4*>(p.out_box)[o] = s_box[c];
    p.out_score[o] = s_score[c];
    p.out_class[o] = s_class[c];
  }
  if (tid == 0) p.out_count[img] = kept;
}

// Dynamic shared memory: scores, boxes, anchors, classes, and the sort order.
constexpr int decode_smem_bytes() {
  return kDecodeMaxAnchors * (4 + 16 + 2 + 1) + 16384 * 2 + 16;
}

// ---------------------------------------------------------------- dense decode
// The reference's InferenceSession.decode_yolo_predictions (runtime/session.py:1223-1278) on the
// GPU: int8 heads -> float32 [B][4 + classes][anchors], anchors level by level. Per anchor:
// dequantize v = (q - zp) * s; per box side a softmax over its 16 bins (max subtracted) and the
// expectation sum_k k * e_k / sum_e; corners (g - d) * stride and (g + d) * stride around the
// grid cell (x, y) (no half-cell offset, as the reference); xywh as centre and size; each class
// 1 / (1 + exp(-v)). One thread per (image, anchor): the head bytes of consecutive anchors are
// consecutive, so the loads and the stores of every output row coalesce. float32 with CUDA's
// expf, against numpy's float32 exp in the reference: equal within a few ulp, not bit for bit.
struct DenseHeadDev {
  long long box_off, cls_off;  // byte offsets inside one image's egress
  float box_scale, box_zp, cls_scale, cls_zp;
  int grid, anchors, anchor_offset;
  float stride;
};
struct DenseParams {
  const int8_t* egress;
  long long egress_image_bytes;
  DenseHeadDev head[3];
  int num_classes, total_anchors;
  float* out;  // [B][4 + num_classes][total_anchors]
};

__global__ void __launch_bounds__(256) dense_decode_kernel(const __grid_constant__ DenseParams p) {
  const int a = blockIdx.x * blockDim.x + threadIdx.x;
  const int img = blockIdx.y;
  if (a >= p.total_anchors) return;
  const int h = a >= p.head[2].anchor_offset ? 2 : (a >= p.head[1].anchor_offset ? 1 : 0);
  const DenseHeadDev& hd = p.head[h];
  const int i = a - hd.anchor_offset, n = hd.anchors;
  const int8_t* eg = p.egress + (long long)img * p.egress_image_bytes;
  const int8_t* box = eg + hd.box_off + i;
  float dist[4];
#pragma unroll
  for (int d = 0; d < 4; ++d) {
    float v[16];
    float m = -FLT_MAX;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      v[k] = __fmul_rn(__fsub_rn((float)box[(long long)(d * 16 + k) * n], hd.box_zp), hd.box_scale);
      m = fmaxf(m, v[k]);
    }
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      v[k] = expf(__fsub_rn(v[k], m));
      sum = __fadd_rn(sum, v[k]);
    }
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) acc = __fadd_rn(acc, __fmul_rn(__fdiv_rn(v[k], sum), (float)k));
    dist[d] = acc;
  }
  const float gx = (float)(i % hd.grid), gy = (float)(i / hd.grid);
  const float x1 = __fmul_rn(__fsub_rn(gx, dist[0]), hd.stride), y1 = __fmul_rn(__fsub_rn(gy, dist[1]), hd.stride);
  const float x2 = __fmul_rn(__fadd_rn(gx, dist[2]), hd.stride), y2 = __fmul_rn(__fadd_rn(gy, dist[3]), hd.stride);
  float* o = p.out + (long long)img * (4 + p.num_classes) * p.total_anchors + a;
  const long long T = p.total_anchors;
  o[0] = __fdiv_rn(__fadd_rn(x1, x2), 2.0f);
  o[T] = __fdiv_rn(__fadd_rn(y1, y2), 2.0f);
  o[2 * T] = __fsub_rn(x2, x1);
  o[3 * T] = __fsub_rn(y2, y1);
  const int8_t* cls = eg + hd.cls_off + i;
  for (int c = 0; c < p.num_classes; ++c) {
    const float v = __fmul_rn(__fsub_rn((float)cls[(long long)c * n], hd.cls_zp), hd.cls_scale);
    o[(4 + c) * T] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v)));
  }
}

}  // namespace ixb
