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
// One CTA decodes one image; its candidates live in shared memory (no scratch in global memory):
//   1. candidates, compacted in anchor order (a block-wide prefix count per 1024 anchors), with the
//      sigmoid tables and, when the DFL exp table depends on q - q_max alone (power-of-two box
//      scales: checked here), its 256-entry diagonal staged in shared memory;
//   2. a stable two-pass radix sort (5-bit digits) of the candidates by score rank, the rank of a
//      score being how many of the three heads' 768 table values exceed it (equal scores, equal
//      ranks): score descending, then anchor ascending, the reference's stable order;
//   3. exact greedy NMS as alternating steps over the list of still-alive candidates (in order,
//      compacted in place after each step): its first 32 are resolved among themselves (any kept
//      box before them has already been applied), then the rest are tested against the step's
//      kept boxes by the whole block, each thread taking a run of consecutive entries, and dropped
//      if one suppresses them. A candidate is dropped only by a kept box ahead of it, and one that
//      reaches a step has survived every kept box ahead of it: the greedy result, in order, with a
//      few block barriers per ~32 kept boxes instead of per 32 candidates.
#pragma once
#include <cfloat>
#include <cstdint>
#include "../../include/ixb200.h"

namespace ixb {

constexpr int kDecodeThreads = 1024;
constexpr int kDecodeCluster = 2;  // CTAs per image (a thread-block cluster)
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
  // Optional, from decode_tables_kernel over the same tables (a session computes them once): the
  // 768 score ranks and, per head, whether the DFL table depends on q - q_max alone. Null: every
  // launch derives them itself.
  const uint16_t* ranks;
  const int32_t* toe;
};

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

// Expectation over the 16 bins of one box side, float32 in the reference's order. `diag` (shared
// memory) holds exp(v(q) - v(q_max)) by q - q_max + 255 when the head's table depends on that
// difference alone; otherwise the table's row q_max is read from global memory.
__device__ __forceinline__ float dfl_side(const int8_t* box, int n, int a, int side, const float* dfl_exp,
                                          const float* diag) {
  int q[kDfl];
  int q_max = -128;
#pragma unroll
  for (int k = 0; k < kDfl; ++k) {
    q[k] = box[(long long)(side * kDfl + k) * n + a];
    q_max = max(q_max, q[k]);
  }
  float e[kDfl];
  if (diag) {
#pragma unroll
    for (int k = 0; k < kDfl; ++k) e[k] = diag[q[k] - q_max + 255];
  } else {
    const float* row = dfl_exp + (q_max + 128) * 256;
#pragma unroll
    for (int k = 0; k < kDfl; ++k) e[k] = __ldg(row + q[k] + 128);
  }
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

__device__ __forceinline__ int warp_incl_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

constexpr int kDecodeWarps = kDecodeThreads / 32;
constexpr int kScoreVals = 3 * 256;   // every score is one of the three heads' sigmoid values
constexpr int kSidxTiny = 0x8000;     // candidate flag: its box area (double) is at most DBL_EPSILON
constexpr int kDecodeMaxPer = (kDecodeMaxAnchors / kDecodeCluster + kDecodeThreads) / kDecodeThreads;  // NMS entries per thread

// Dynamic shared memory of the decode kernel (byte offsets).
constexpr int kDsBox = 0;                                   // float4 [8400]: x0, y0, w, h
constexpr int kDsSidx = kDsBox + 16 * kDecodeMaxAnchors;    // uint16 [8400]: head * 256 + q + 128 | tiny
constexpr int kDsCls = kDsSidx + 2 * kDecodeMaxAnchors;     // uint8 [8400]: class
constexpr int kDsOrdA = kDsCls + kDecodeMaxAnchors;         // uint16 [8400]: sort buffers; A ends sorted,
constexpr int kDsOrdB = kDsOrdA + 2 * kDecodeMaxAnchors;    //   B then holds the kept list
constexpr int kDsSig = kDsOrdB + 2 * kDecodeMaxAnchors;     // float [768]: sigmoid tables
constexpr int kDsDiag = kDsSig + 4 * kScoreVals;            // float [768]: DFL exp diagonals
constexpr int kDsLow = kDsDiag + 4 * kScoreVals;            // int32 [768]: sigmoid_low tables
constexpr int kDsRank = kDsLow + 4 * kScoreVals;            // uint16 [768]: score ranks
constexpr int kDsWc = kDsRank + 2 * kScoreVals;             // int [32][33]: per-warp counts
constexpr int kDsBytes = kDsWc + 4 * 32 * 33;

// One stable counting pass over 32 buckets: dst[start(d) + earlier entries of digit d] = src[i].
// Entries go 1024 at a time; a warp's entries of one digit find each other with match.any, and
// a transposed warp scan (warp d over the 32 warps' counts of digit d) places the warps in order.
// s_wc must be zero on entry and is zero again on exit.
template <typename Digit>
__device__ __forceinline__ void radix_pass(const uint16_t* src, uint16_t* dst, int n, Digit digit, int* s_cnt,
                                           int (*s_wc)[33], int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  if (tid < 32) s_cnt[tid] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += kDecodeThreads) atomicAdd(&s_cnt[digit(src[i])], 1);
  __syncthreads();
  if (warp == 0) {
    const int v = s_cnt[lane];
    s_cnt[lane] = warp_incl_scan(v, lane) - v;  // where each digit's run starts
  }
  __syncthreads();
  for (int base = 0; base < n; base += kDecodeThreads) {
    const int i = base + tid;
    const bool valid = i < n;
    const uint16_t key = valid ? src[i] : (uint16_t)0;
    const int d = valid ? digit(key) : 32;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int below = __popc(peers & ((1u << lane) - 1u));
    if (valid && below == 0) s_wc[warp][d] = __popc(peers);
    __syncthreads();
    {  // warp `warp` places digit `warp`: the 32 warps' counts in warp order after the digit's run so far
      const int v = s_wc[lane][warp];
      const int run = s_cnt[warp];
      const int incl = warp_incl_scan(v, lane);
      s_wc[lane][warp] = run + incl - v;
      __syncwarp();
      if (lane == 31) s_cnt[warp] = run + incl;
    }
    __syncthreads();
    if (valid) dst[s_wc[warp][d] + below] = key;
    __syncwarp();
    s_wc[warp][lane] = 0;
    __syncthreads();
  }
}

// Whether the cross-class pair (i, k) cannot overlap after the class offsets: the box of the
// higher class lies right of the other's by at least a pixel whenever its x0 >= 0 (classes one
// apart) or x0 >= -(gap - 1) * max_coord (further apart), every box ending at or before max_coord.
// Then the intersection is 0 and, unless both areas are at most DBL_EPSILON, the overlap is 0,
// which suppresses nothing for an IoU threshold >= 0 (the caller checks).
__device__ __forceinline__ bool classes_apart(float4 bi, int ci, float4 bk, int ck, double maxc) {
  if (ci == ck) return false;
  const float x_hi = ci < ck ? bk.x : bi.x;
  const int gap = ci < ck ? ck - ci : ci - ck;
  return x_hi >= 0.f || (double)x_hi >= -(double)(gap - 1) * maxc;
}

// The suppression test of two boxes of one class decided in float, when the float overlap
// measure d = inter - iou * union is farther from 0 than its rounding can move it: 1 (suppresses),
// 0 (does not), -1 (too close: the exact test decides). Same class, same offset: the exact test's
// double arithmetic on offset coordinates is the exact arithmetic of the raw float coordinates
// (to ~1e-16). Each float rounding moves a result by at most 2^-24 of its magnitude; with M the
// largest coordinate magnitude of the pair, the side lengths of the intersection are off by at
// most delta = 2^-22 M, the intersection by delta * P + delta^2 + 2^-24 inter (P the sum of the
// four sides), and d by at most err = 2 delta P + 2 delta^2 + 2^-21 (areas + union + inter). The
// exact test suppresses when d / union > 1e-6 and keeps when d / union < -1e-6 (its float
// roundings of the overlap are ~1e-7), so |d| > err + 2e-6 union decides. iou in [0, 1].
__device__ __forceinline__ int screen_same_class(float4 a, float4 b, float iou) {
  const float ax2 = a.x + a.z, ay2 = a.y + a.w, bx2 = b.x + b.z, by2 = b.y + b.w;
  const float iw = fminf(ax2, bx2) - fmaxf(a.x, b.x);
  const float ih = fminf(ay2, by2) - fmaxf(a.y, b.y);
  const float inter = (iw > 0.f && ih > 0.f) ? iw * ih : 0.f;
  const float aa = a.z * a.w, ab = b.z * b.w;
  const float uni = (aa + ab) - inter;
  const float m = fmaxf(fmaxf(fmaxf(fabsf(a.x), fabsf(ax2)), fmaxf(fabsf(a.y), fabsf(ay2))),
                        fmaxf(fmaxf(fabsf(b.x), fabsf(bx2)), fmaxf(fabsf(b.y), fabsf(by2))));
  const float delta = m * 2.384185791015625e-7f;  // 2^-22
  const float per = (a.z + a.w) + (b.z + b.w);
  const float err = 2.f * delta * (per + delta) + 4.76837158203125e-7f * (aa + ab + uni + inter);  // 2^-21
  const float margin = err + 2e-6f * uni;
  const float d = inter - iou * uni;
  if (d > margin) return 1;
  if (d < -margin) return 0;
  return -1;  // near the threshold, or not finite
}

// Whether kept box k suppresses candidate i: classes that cannot meet after the offsets and clear
// same-class cases are decided without the exact double test.
__device__ __forceinline__ bool pair_suppresses(float4 bi, int cli, bool tiny_i, float4 bk, int clk, bool tiny_k,
                                                double off_step, double maxc, float iou, bool iou_nonneg,
                                                bool iou_unit) {
  if (iou_nonneg && !(tiny_i && tiny_k)) {
    if (cli != clk) {
      if (classes_apart(bi, cli, bk, clk, maxc)) return false;
    } else if (iou_unit) {
      const int r = screen_same_class(bi, bk, iou);
      if (r >= 0) return r != 0;
    }
  }
  return suppresses(bi, __dmul_rn((double)cli, off_step), bk, __dmul_rn((double)clk, off_step), iou);
}

__global__ void __launch_bounds__(kDecodeThreads, 1) yolo_decode_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(16) uint8_t dsmem[];
  float4* s_box = reinterpret_cast<float4*>(dsmem + kDsBox);
  uint16_t* s_sidx = reinterpret_cast<uint16_t*>(dsmem + kDsSidx);
  uint8_t* s_class = dsmem + kDsCls;
  uint16_t* s_ordA = reinterpret_cast<uint16_t*>(dsmem + kDsOrdA);
  uint16_t* s_ordB = reinterpret_cast<uint16_t*>(dsmem + kDsOrdB);
  float* s_sig = reinterpret_cast<float*>(dsmem + kDsSig);
  float* s_diag = reinterpret_cast<float*>(dsmem + kDsDiag);
  int32_t* s_low = reinterpret_cast<int32_t*>(dsmem + kDsLow);
  uint16_t* s_rank = reinterpret_cast<uint16_t*>(dsmem + kDsRank);
  int(*s_wc)[33] = reinterpret_cast<int(*)[33]>(dsmem + kDsWc);
  __shared__ int s_n, s_kept, s_nv, s_nk, s_L;
  __shared__ int s_pc[2][kDecodeCluster];  // per-rank counts traded each round (double-buffered by parity)
  __shared__ float4 s_nkbox[32];  // the current step's kept boxes, their classes and tiny flags
  __shared__ int s_nkcls[32], s_nktiny[32];
  __shared__ int s_cnt[32], s_wcnt[kDecodeWarps];
  __shared__ int s_toe[3], s_toe_half[kDecodeCluster][3];
  __shared__ double s_maxc[kDecodeWarps];

  __shared__ unsigned s_mask[32];

  const int img = blockIdx.x / kDecodeCluster, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t crank = cluster_rank(), cpeer = crank ^ 1u;
  const int8_t* eg = p.egress + (long long)img * p.egress_image_bytes;
  const float pad_top = p.letterbox[3 * img], pad_left = p.letterbox[3 * img + 1], lscale = p.letterbox[3 * img + 2];
  const int total = p.head[0].anchors + p.head[1].anchors + p.head[2].anchors;

  // 0. tables: sigmoid values (and the first index of each value's run), the DFL diagonals
  for (int i = tid; i < kScoreVals; i += kDecodeThreads) {
    const DecodeHeadDev& hd = p.head[i >> 8];
    s_sig[i] = __ldg(hd.sigmoid + (i & 255));
    s_low[i] = hd.sigmoid_low ? __ldg(hd.sigmoid_low + (i & 255)) : 0;
    s_diag[i] = __ldg(hd.dfl_exp + 255 * 256 + (i & 255));  // row q_max = 127
  }
  if (tid == 0) {
    s_n = 0;
    s_kept = 0;
  }
  if (p.ranks) {
    for (int i = tid; i < kScoreVals; i += kDecodeThreads) s_rank[i] = __ldg(p.ranks + i);
    if (tid < 3) s_toe[tid] = __ldg(p.toe + tid);
    cluster_sync();  // both CTAs of the cluster are running before either touches the other's shared memory
  } else {
    cluster_sync();  // both CTAs of the cluster are running before either touches the other's shared memory
    // The image's two CTAs split the checks and the ranks (rows and values of their own parity) and
    // trade the results.
    for (int h = 0; h < 3; ++h) {
      // the table is used at (q_max, q) with q <= q_max only: there it must equal the diagonal
      // (16-byte loads of four columns; the caller's tables are 16-byte aligned)
      const float4* t4 = reinterpret_cast<const float4*>(p.head[h].dfl_exp);
      const float* dg = s_diag + h * 256 + 255;
      bool same = true;
#pragma unroll 4
      for (int e = tid; e < 128 * 64; e += kDecodeThreads) {
        const int r = 2 * (e >> 6) + (int)crank, c = (e & 63) * 4;
        if (c <= r) {
          const float4 v = __ldg(t4 + r * 64 + (e & 63));
          same &= __float_as_uint(v.x) == __float_as_uint(dg[c - r]);
          same &= c + 1 > r || __float_as_uint(v.y) == __float_as_uint(dg[c + 1 - r]);
          same &= c + 2 > r || __float_as_uint(v.z) == __float_as_uint(dg[c + 2 - r]);
          same &= c + 3 > r || __float_as_uint(v.w) == __float_as_uint(dg[c + 3 - r]);
        }
      }
      same = __syncthreads_and(same) != 0;
      if (tid == 0) {
        s_toe_half[crank][h] = same ? 1 : 0;
        st_cluster_u32(cluster_addr(&s_toe_half[crank][h], cpeer), same ? 1u : 0u);
      }
    }
    for (int i = 2 * tid + (int)crank; i < kScoreVals; i += 2 * kDecodeThreads) {
      const float v = s_sig[i];
      int r = 0;
      for (int j = 0; j < kScoreVals; ++j) r += s_sig[j] > v ? 1 : 0;
      s_rank[i] = (uint16_t)r;
      st_cluster_u16(cluster_addr(&s_rank[i], cpeer), (uint32_t)r);
    }
    cluster_sync();  // both halves of the checks and of the ranks in both CTAs
    if (tid < 3) s_toe[tid] = s_toe_half[0][tid] & s_toe_half[1][tid];
    __syncthreads();
  }

  // 1. candidates in anchor order: prune, class score, DFL, box. The image's two CTAs take
  //    alternate 1024-anchor tiles; after each pair they trade counts, and each writes its
  //    candidates into both CTAs' arrays at their places in anchor order.
  int it = 0;
  for (int base = 0; base < total; base += kDecodeThreads * kDecodeCluster, ++it) {
    const int A = base + (int)crank * kDecodeThreads + tid;
    bool pass = false;
    float4 bx = make_float4(0.f, 0.f, 0.f, 0.f);
    int sidx = 0, best_c = 0;
    if (A < total) {
      const int h = (A >= p.head[1].anchor_offset) + (A >= p.head[2].anchor_offset);
      const DecodeHeadDev& hd = p.head[h];
      const int n = hd.anchors, a = A - hd.anchor_offset;
      const int8_t* box = eg + hd.box_off;
      const int8_t* cls = eg + hd.cls_off;
      int q_max = -128, c_max = 0;  // the maximum byte and the first class holding it
#pragma unroll 16
      for (int c = 0; c < p.num_classes; ++c) {
        const int q = cls[(long long)c * n + a];
        if (q > q_max) {
          q_max = q;
          c_max = c;
        }
      }
      if (q_max > hd.qi) {
        const float* sig = s_sig + h * 256 + 128;
        float best;
        int q_best = q_max;
        if (hd.sigmoid_low) {
          best = sig[q_max];
          pass = best >= p.conf;
          if (pass) {
            // the first class whose byte reaches lo, the lowest byte with q_max's sigmoid value:
            // c_max when no smaller byte shares that value (the usual case, without a walk
            // through the class bytes)
            const int lo = s_low[h * 256 + q_max + 128];
            if (lo == q_max) {
              best_c = c_max;
            } else {
              while (best_c < p.num_classes - 1 && (int)cls[(long long)best_c * n + a] < lo) ++best_c;
            }
          }
        } else {
          q_best = cls[a];
          best = sig[q_best];
          for (int c = 1; c < p.num_classes; ++c) {
            const int q = cls[(long long)c * n + a];
            const float pr = sig[q];
            if (pr > best) {
              best = pr;
              best_c = c;
              q_best = q;
            }
          }
          pass = best >= p.conf;
        }
        if (pass) {
          const float* diag = s_toe[h] ? s_diag + h * 256 : nullptr;
          const float l = dfl_side(box, n, a, 0, hd.dfl_exp, diag);
          const float t = dfl_side(box, n, a, 1, hd.dfl_exp, diag);
          const float r = dfl_side(box, n, a, 2, hd.dfl_exp, diag);
          const float b = dfl_side(box, n, a, 3, hd.dfl_exp, diag);
          const float ax = __ldg(p.anchor_x + A), ay = __ldg(p.anchor_y + A), st = __ldg(p.strides + A);
          const float x1 = __fsub_rn(ax, l), y1 = __fsub_rn(ay, t), x2 = __fadd_rn(ax, r), y2 = __fadd_rn(ay, b);
          const float cx = __fmul_rn(__fmul_rn(__fadd_rn(x1, x2), 0.5f), st);
          const float cy = __fmul_rn(__fmul_rn(__fadd_rn(y1, y2), 0.5f), st);
          const float bw = __fmul_rn(__fsub_rn(x2, x1), st);
          const float bh = __fmul_rn(__fsub_rn(y2, y1), st);
          bx = make_float4(__fdiv_rn(__fsub_rn(__fsub_rn(cx, __fdiv_rn(bw, 2.0f)), pad_left), lscale),
                           __fdiv_rn(__fsub_rn(__fsub_rn(cy, __fdiv_rn(bh, 2.0f)), pad_top), lscale),
                           __fdiv_rn(bw, lscale), __fdiv_rn(bh, lscale));
          sidx = h * 256 + q_best + 128;
          if (__dmul_rn((double)bx.z, (double)bx.w) <= DBL_EPSILON) sidx |= kSidxTiny;
        }
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, pass);
    if (lane == 0) s_wcnt[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
      const int v = s_wcnt[lane];
      const int incl = warp_incl_scan(v, lane);
      s_wcnt[lane] = incl - v;
      if (lane == 31) {
        s_pc[it & 1][crank] = incl;
        st_cluster_u32(cluster_addr(&s_pc[it & 1][crank], cpeer), (uint32_t)incl);
      }
    }
    cluster_sync();  // both tiles' counts in both CTAs
    const int c0 = s_pc[it & 1][0], c1 = s_pc[it & 1][1];
    if (pass) {
      const int slot = s_n + (crank ? c0 : 0) + s_wcnt[warp] + __popc(bal & ((1u << lane) - 1u));
      s_box[slot] = bx;
      s_sidx[slot] = (uint16_t)sidx;
      s_class[slot] = (uint8_t)best_c;
      st_cluster_f4(cluster_addr(&s_box[slot], cpeer), bx);
      st_cluster_u16(cluster_addr(&s_sidx[slot], cpeer), (uint32_t)sidx);
      st_cluster_u8(cluster_addr(&s_class[slot], cpeer), (uint32_t)best_c);
    }
    __syncthreads();
    if (tid == 0) s_n += c0 + c1;
    __syncthreads();
  }
  cluster_sync();  // every candidate, written by either CTA, is in both
  const int n = s_n;
  if (n == 0) {
    if (tid == 0 && crank == 0) p.out_count[img] = 0;
    return;
  }

  // 2. the class offset of NMSBoxesBatched (max over every candidate's corners, starting at 0), and
  //    the order: score descending (rank ascending), then anchor ascending (slot order)
  double mc = 0.0;
  for (int i = tid; i < n; i += kDecodeThreads) {
    const float4 b = s_box[i];
    const double x1 = b.x, y1 = b.y, x2 = __dadd_rn(x1, (double)b.z), y2 = __dadd_rn(y1, (double)b.w);
    mc = fmax(mc, fmax(fmax(x1, y1), fmax(x2, y2)));
    s_ordA[i] = (uint16_t)i;
  }
  for (int o = 16; o > 0; o >>= 1) mc = fmax(mc, __shfl_xor_sync(0xffffffffu, mc, o));
  if (lane == 0) s_maxc[warp] = mc;
  s_wc[warp][lane] = 0;
  if (lane == 0) s_wc[warp][32] = 0;
  __syncthreads();
  radix_pass(s_ordA, s_ordB, n, [&](uint16_t k) { return (int)(s_rank[s_sidx[k] & 0x3FF] & 31); }, s_cnt, s_wc, tid);
  radix_pass(s_ordB, s_ordA, n, [&](uint16_t k) { return (int)(s_rank[s_sidx[k] & 0x3FF] >> 5); }, s_cnt, s_wc, tid);
  double maxc = 0.0;
  for (int w = 0; w < kDecodeWarps; ++w) maxc = fmax(maxc, s_maxc[w]);
  const double off_step = __dadd_rn(maxc, 1.0);
  const bool iou_nonneg = p.iou >= 0.f;  // false for NaN too
  const bool iou_unit = iou_nonneg && p.iou <= 1.f;

  // 3. NMS. Scores strictly above conf are a prefix of the order; s_ordA[0, L) then holds the
  //    alive candidates in order, compacted in place after every step.
  if (tid == 0) s_nv = n;
  __syncthreads();
  for (int i = tid; i < n; i += kDecodeThreads)
    if (!(s_sig[s_sidx[s_ordA[i]] & 0x3FF] > p.conf)) atomicMin(&s_nv, i);
  __syncthreads();
  const int nv = s_nv;
  if (tid == 0) s_L = nv;
  __syncthreads();
  for (int step = 0; step < nv; ++step) {  // each step takes at least one alive candidate
    const int L = s_L;
    const int cn = min(32, L);
    if (cn == 0) break;
    // a. the chunk s_ordA[0, cn) among itself: does earlier member b suppress member a (warp a, lane b)
    if (warp < cn) {
      const uint16_t ca = s_ordA[warp];
      const float4 ba = s_box[ca];
      const int cla = s_class[ca];
      const bool tiny_a = (s_sidx[ca] & kSidxTiny) != 0;
      bool m = false;
      if (lane < warp) {
        const uint16_t cb = s_ordA[lane];
        m = pair_suppresses(ba, cla, tiny_a, s_box[cb], s_class[cb], (s_sidx[cb] & kSidxTiny) != 0, off_step, maxc,
                            p.iou, iou_nonneg, iou_unit);
      }
      const unsigned mask = __ballot_sync(0xffffffffu, m);
      if (lane == 0) s_mask[warp] = mask;
    }
    __syncthreads();
    if (warp == 0) {
      unsigned keep = 0u;
      for (int a = 0; a < cn; ++a)
        if (!(s_mask[a] & keep)) keep |= 1u << a;
      const int kept = s_kept;
      if ((keep >> lane) & 1u) {
        const int r = __popc(keep & ((1u << lane) - 1u));
        const uint16_t c = s_ordA[lane];
        s_ordB[kept + r] = c;
        s_nkbox[r] = s_box[c];
        s_nkcls[r] = s_class[c];
        s_nktiny[r] = (s_sidx[c] & kSidxTiny) != 0 ? 1 : 0;
      }
      if (lane == 0) {
        s_kept = kept + __popc(keep);
        s_nk = __popc(keep);
      }
    }
    __syncthreads();
    // b. the rest, s_ordA[cn, L), against the chunk's kept boxes: the image's two CTAs take one
    //    half each, thread t a run of E consecutive entries of it (E <= 5) held in registers; the
    //    survivors are written back in order into both CTAs' lists
    const int nk = s_nk, rest = L - cn, half = (rest + 1) / 2;
    const int lo = cn + (crank ? half : 0), hi = crank ? L : cn + half;
    const int E = (hi - lo + kDecodeThreads - 1) / kDecodeThreads, i0 = lo + tid * E;
    uint32_t cid[kDecodeMaxPer];
    unsigned live = 0u;
#pragma unroll
    for (int e = 0; e < kDecodeMaxPer; ++e) {
      cid[e] = 0u;
      if (e < E && i0 + e < hi) {
        const uint16_t ci = s_ordA[i0 + e];
        cid[e] = ci;
        const float4 bi = s_box[ci];
        const int cli = s_class[ci];
        const bool tiny_i = (s_sidx[ci] & kSidxTiny) != 0;
        bool alive = true;
        for (int j = 0; j < nk && alive; ++j)
          if (pair_suppresses(bi, cli, tiny_i, s_nkbox[j], s_nkcls[j], s_nktiny[j] != 0, off_step, maxc, p.iou,
                              iou_nonneg, iou_unit))
            alive = false;
        if (alive) live |= 1u << e;
      }
    }
    const int cnt = __popc(live);
    int incl = warp_incl_scan(cnt, lane);
    if (lane == 31) s_wcnt[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int v = s_wcnt[lane];
      const int wi = warp_incl_scan(v, lane);
      s_wcnt[lane] = wi - v;
      if (lane == 31) {
        s_pc[step & 1][crank] = wi;
        st_cluster_u32(cluster_addr(&s_pc[step & 1][crank], cpeer), (uint32_t)wi);
      }
    }
    cluster_sync();  // both halves' counts here, and every entry of both CTAs read before any is overwritten
    const int t0 = s_pc[step & 1][0], t1 = s_pc[step & 1][1];
    int dst = (crank ? t0 : 0) + s_wcnt[warp] + incl - cnt;
#pragma unroll
    for (int e = 0; e < kDecodeMaxPer; ++e)
      if ((live >> e) & 1u) {
        s_ordA[dst] = (uint16_t)cid[e];
        st_cluster_u16(cluster_addr(&s_ordA[dst], cpeer), cid[e]);
        ++dst;
      }
    if (tid == 0) s_L = t0 + t1;
    cluster_sync();  // the new list in both CTAs
  }

  // 4. detections in kept order
  const int kept = s_kept;
  if (crank != 0) return;  // both CTAs hold the same result
  if (kept > p.capacity) {
    if (tid == 0) p.out_count[img] = -3;
    return;
  }
  for (int k = tid; k < kept; k += kDecodeThreads) {
    const uint16_t c = s_ordB[k];
    const long long o = (long long)img * p.capacity + k;
    reinterpret_cast<float4*>(p.out_box)[o] = s_box[c];
    p.out_score[o] = s_sig[s_sidx[c] & 0x3FF];
    p.out_class[o] = s_class[c];
  }
  if (tid == 0) p.out_count[img] = kept;
}

constexpr int decode_smem_bytes() { return kDsBytes; }

// The per-table part of the decode, once for a set of tables (one CTA of kDecodeThreads): each
// score value's rank (how many of the three heads' 768 sigmoid values exceed it) and, per head,
// whether the DFL exp table equals its q_max = 127 row's diagonal wherever the decode reads it
// (q <= q_max). The same tests as the decode kernel's own, over every row.
__global__ void __launch_bounds__(kDecodeThreads, 1) decode_tables_kernel(const __grid_constant__ DecodeParams p,
                                                                          uint16_t* ranks, int32_t* toe) {
  __shared__ float s_sig[kScoreVals], s_diag[kScoreVals];
  const int tid = threadIdx.x;
  for (int i = tid; i < kScoreVals; i += kDecodeThreads) {
    const DecodeHeadDev& hd = p.head[i >> 8];
    s_sig[i] = __ldg(hd.sigmoid + (i & 255));
    s_diag[i] = __ldg(hd.dfl_exp + 255 * 256 + (i & 255));
  }
  __syncthreads();
  for (int h = 0; h < 3; ++h) {
    const float4* t4 = reinterpret_cast<const float4*>(p.head[h].dfl_exp);
    const float* dg = s_diag + h * 256 + 255;
    bool same = true;
    for (int e = tid; e < 256 * 64; e += kDecodeThreads) {
      const int r = e >> 6, c = (e & 63) * 4;
      if (c <= r) {
        const float4 v = __ldg(t4 + r * 64 + (e & 63));
        same &= __float_as_uint(v.x) == __float_as_uint(dg[c - r]);
        same &= c + 1 > r || __float_as_uint(v.y) == __float_as_uint(dg[c + 1 - r]);
        same &= c + 2 > r || __float_as_uint(v.z) == __float_as_uint(dg[c + 2 - r]);
        same &= c + 3 > r || __float_as_uint(v.w) == __float_as_uint(dg[c + 3 - r]);
      }
    }
    same = __syncthreads_and(same) != 0;
    if (tid == 0) toe[h] = same ? 1 : 0;
  }
  for (int i = tid; i < kScoreVals; i += kDecodeThreads) {
    const float v = s_sig[i];
    int r = 0;
    for (int j = 0; j < kScoreVals; ++j) r += s_sig[j] > v ? 1 : 0;
    ranks[i] = (uint16_t)r;
  }
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
