// libixb200.so: the C ABI of include/ixb200.h over the sm_100a kernels.
//
// The host side checks every descriptor before anything launches: each view a kernel reads
// or writes must lie inside the arena for the batch size used, with the alignment the
// 16-byte copies and stores need. A session replays one captured CUDA graph per batch size
// (input staging -> image ingress -> every layer -> head egress) on its own stream.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <utility>
#include <vector>

#include "../../include/ixb200.h"
#include "ixb_conv.cuh"
#include "ixb_decode.cuh"
#include "ixb_gemm.cuh"
#include "ixb_misc.cuh"
#include "ixb_w4a8.cuh"
#include "ixb_ptx.cuh"

using namespace ixb;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(IXB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define IXB_CUDA(call)                                      \
  do {                                                      \
    cudaError_t e_ = (call);                                \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call);     \
  } while (0)

constexpr int kSmemLimit = 227 * 1024;
constexpr int kConvDynSmem = kSmemLimit - 256;  // the conv kernel holds its 256-byte table statically

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// Raises a kernel's dynamic shared-memory limit once per (kernel, device): cudaFuncSetAttribute
// applies to the current device's context only, so a process with sessions on several GPUs sets
// it on each. Kernels of one signature share a function-pointer type, so the key is the address.
template <typename Kern>
int ensure_smem_limit(Kern kern, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  IXB_CUDA(cudaGetDevice(&dev));
  const std::pair<const void*, int> key(reinterpret_cast<const void*>(kern), dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return 0;
  IXB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert(key);
  return 0;
}

// SMs the launch planner spreads tiles over: the current device's count (148 on B200), 148
// when no device answers (host-side checks run without a GPU), or IXB_SM_COUNT when set
// (tests use it to force the multi-block tiles on small inputs).
int sm_count() {
  if (const char* env = getenv("IXB_SM_COUNT")) {
    const int v = atoi(env);
    if (v > 0) return v;
  }
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

// A view touches, for `batch` images, every chunk plane it names from `guard` pixels before the
// first image to `guard` pixels after the last; all of it must lie inside the arena, the planes
// must not overlap, and the 16-byte copies need 16-byte alignment. The image tensor is one plane
// of 8-byte pixels [batch][H+2][W+4].
int check_seg(const ixb_segment& s, int batch, uint64_t arena_bytes, bool image, const char* what,
              std::string& err) {
  char buf[256];
  if (s.height < 1 || s.width < 1 || s.channels < 1 || s.chunk_offset < 0 || s.guard < 0) {
    snprintf(buf, sizeof buf, "%s: empty or negative view", what);
    err = buf;
    return -1;
  }
  if (image) {
    const unsigned long long bytes = (unsigned long long)batch * (s.height + 2) * (unsigned long long)(s.width + 4) * 8;
    if (s.channels != 3 || s.chunk_offset || s.guard || s.offset % 16 || s.width % 2 || s.offset + bytes > arena_bytes) {
      snprintf(buf, sizeof buf, "%s: the image tensor is one guard-free plane of 8-byte pixels inside the arena",
               what);
      err = buf;
      return -1;
    }
    return 0;
  }
  const unsigned long long pix = (unsigned long long)batch * (s.height + 2) * (unsigned long long)(s.width + 2);
  if (s.channels % 16 || s.offset % 16 || s.plane_stride % 16) {
    snprintf(buf, sizeof buf, "%s: misaligned view (offset %llu plane %llu channels %d)", what,
             (unsigned long long)s.offset, (unsigned long long)s.plane_stride, s.channels);
    err = buf;
    return -1;
  }
  const unsigned long long nch = s.channels / 16;
  if (nch > 1 && s.plane_stride < (pix + 2ull * s.guard) * 16) {
    snprintf(buf, sizeof buf, "%s: chunk planes overlap", what);
    err = buf;
    return -1;
  }
  const unsigned long long first = (unsigned long long)s.chunk_offset * s.plane_stride;
  if (s.offset + first < 16ull * s.guard ||
      s.offset + first + (nch - 1) * s.plane_stride + (pix + s.guard) * 16 > arena_bytes) {
    snprintf(buf, sizeof buf, "%s: view reaches outside the %llu-byte arena", what, (unsigned long long)arena_bytes);
    err = buf;
    return -1;
  }
  return 0;
}

SegDev seg_dev(const ixb_segment& s, uint8_t* arena, int chunk_begin) {
  SegDev d;
  d.base = reinterpret_cast<const int8_t*>(arena + s.offset + (uint64_t)s.chunk_offset * s.plane_stride);
  d.plane = (long long)s.plane_stride;
  d.chunk_begin = chunk_begin;
  d.chunks = (s.channels + 15) / 16;
  d.H = s.height;
  d.W = s.width;
  d.up2 = s.up2;
  d.P = (s.height + 2) * (s.width + 2);
  const long long img_bytes = (long long)d.P * 16;
  d.plane_images = (s.plane_stride && s.plane_stride % img_bytes == 0) ? (int)(s.plane_stride / img_bytes) : 0;
  return d;
}

// K schedule of a conv: the K-blocks (A slots, MMAs, weights) and per MMA the (slot, chunk, tap)
// of its two 32-byte K-halves. The weight packer (ignite_xdna_b200/plan.py) lays B out in exactly
// this order. Slot s of a K-block holds chunk chunk0 + s / ntaps at tap tap0 + s % ntaps.
//  WINDOW: full chunk pairs, cp pairs per K-block, all taps as window shifts of the pair's slots;
//          an odd last chunk gets a K-block whose MMAs pair consecutive taps of that chunk.
//  IM2COL: K-blocks per (image row ky, group of cp full pairs) holding the loaded taps kx = 0, 1 of
//          each chunk (slot = chunk * 2 + kx) and the MMAs of kx = 0, 1, 2 (kx = 2 reads the kx = 0
//          slot one row on); an odd last chunk gets one K-block of its six loaded taps.
//  GATHER: K-blocks over groups of cp pairs (1x1); a missing second chunk is a zero-weight half.
//  STEM:   one K-block of three slots, one per image row ky; tap 2 * ky + p is pixel pair p of that
//          row, pair 1 read as the slot one row on.
struct SchedKB {
  int chunk0, nchunks, tap0, ntaps, op0, nops, b_off, b_bytes;
};
struct SchedOp {
  int slot0, chunk0, tap0, slot1, chunk1, tap1;  // chunk1 < 0: the second half multiplies zero weights
};

int build_schedule(const ixb_conv_desc& d, int cin_chunks, std::vector<SchedKB>& kbs, std::vector<SchedOp>& ops) {
  kbs.clear();
  ops.clear();
  const int taps = d.k * d.k;
  const int opb = d.n_tile * 32;
  int b_off = 0;
  auto push_kb = [&](int chunk0, int nchunks, int tap0, int ntaps, int op0) {
    const int nops = (int)ops.size() - op0;
    kbs.push_back(SchedKB{chunk0, nchunks, tap0, ntaps, op0, nops, b_off, nops * opb});
    b_off += nops * opb;
  };
  const int E = cin_chunks / 2, odd = cin_chunks % 2;
  if (d.mode == IXB_MODE_STEM) {
    // slot ky holds image row ky; the MMA's two K-halves are pairs 0 and 1 of that row (tap 2ky+p),
    // the second read one row on in the same slot
    for (int ky = 0; ky < 3; ++ky) ops.push_back(SchedOp{ky, 0, 2 * ky, ky, 0, 2 * ky + 1});
    push_kb(0, 1, 0, 3, 0);
  } else if (d.mode == IXB_MODE_WINDOW && d.s2d_in == 1) {
    // Space-to-depth view of a stride-2 3x3 conv: chunk c is phase (ry, rx) = (p / 2, p % 2),
    // p = c / (cin_chunks / 4); tap t of the 2x2 is (dy, dx) = (t / 2 - 1, t % 2 - 1). Output (y, x)
    // tap (ky, kx) of the 3x3 reads input (2y + ky - 1, 2x + kx - 1): phase 1 one pixel back for
    // k = 0, phase 0 for k = 1, phase 1 for k = 2, so a (chunk, tap) pair carries weights unless
    // it reaches back (d = -1) in a phase-0 direction. Per K-block of 2 cp chunks, the valid pairs
    // are ordered by their A address (slot, then shift) and paired into MMAs, an odd one with a
    // zero half: 9 of 16 pairs, the 3x3's own K.
    const int C = cin_chunks / 4;
    auto valid = [&](int c, int t) {
      const int ph = c / C, ry = ph / 2, rx = ph % 2;
      return !((t / 2 == 0 && ry == 0) || (t % 2 == 0 && rx == 0));
    };
    const int sh[4] = {0, 1, d.in_w + 2, d.in_w + 3};
    for (int g = 0; g * d.cp < E; ++g) {
      const int prs = std::min(d.cp, E - g * d.cp), op0 = (int)ops.size(), c0 = 2 * g * d.cp;
      std::vector<std::pair<long long, std::pair<int, int>>> halves;  // (address, (slot, tap))
      for (int sl = 0; sl < 2 * prs; ++sl)
        for (int t = 0; t < 4; ++t)
          if (valid(c0 + sl, t)) halves.push_back({(long long)sl * (1LL << 40) + sh[t], {sl, t}});
      std::sort(halves.begin(), halves.end());
      for (size_t i = 0; i < halves.size(); i += 2) {
        const int s0 = halves[i].second.first, t0 = halves[i].second.second;
        if (i + 1 < halves.size()) {
          const int s1 = halves[i + 1].second.first, t1 = halves[i + 1].second.second;
          ops.push_back(SchedOp{s0, c0 + s0, t0, s1, c0 + s1, t1});
        } else {
          ops.push_back(SchedOp{s0, c0 + s0, t0, 0, -1, 0});
        }
      }
      push_kb(c0, 2 * prs, 0, 1, op0);
    }
  } else if (d.mode == IXB_MODE_WINDOW) {
    for (int g = 0; g * d.cp < E; ++g) {
      const int prs = std::min(d.cp, E - g * d.cp), op0 = (int)ops.size(), c0 = 2 * g * d.cp;
      for (int i = 0; i < prs; ++i)
        for (int t = 0; t < taps; ++t) ops.push_back(SchedOp{2 * i, c0 + 2 * i, t, 2 * i + 1, c0 + 2 * i + 1, t});
      push_kb(c0, 2 * prs, 0, 1, op0);
    }
    if (odd) {
      const int op0 = (int)ops.size();
      for (int t = 0; t < taps; t += 2)
        ops.push_back(t + 1 < taps ? SchedOp{0, 2 * E, t, 0, 2 * E, t + 1} : SchedOp{0, 2 * E, t, 0, -1, 0});
      push_kb(2 * E, 1, 0, 1, op0);
    }
  } else if (d.mode == IXB_MODE_IM2COL) {
    // Loaded taps: kx = 0 and 1 of each image row ky (loaded tap 2 ky + kx); kx = 2 of output x is
    // kx = 0 of output x + 1, read as the kx = 0 slot one row on. Per (ky, chunk group) a K-block
    // holds both loaded taps of its chunks and the MMAs of all three kx.
    for (int ky = 0; ky < 3; ++ky) {
      for (int g = 0; g * d.cp < E; ++g) {
        const int prs = std::min(d.cp, E - g * d.cp), op0 = (int)ops.size(), c0 = 2 * g * d.cp;
        for (int kx = 0; kx < 3; ++kx) {
          const int t = 3 * ky + kx, lx = kx == 2 ? 0 : kx;
          for (int i = 0; i < prs; ++i)
            ops.push_back(SchedOp{2 * (2 * i) + lx, c0 + 2 * i, t, 2 * (2 * i + 1) + lx, c0 + 2 * i + 1, t});
        }
        push_kb(c0, 2 * prs, 2 * ky, 2, op0);
      }
    }
    if (odd) {
      // the last chunk alone: its six loaded taps in one K-block, consecutive taps paired
      // (an MMA's second K-half must lie above its first: halves are ordered by slot, then shift)
      auto slot_of = [](int t) { return 2 * (t / 3) + (t % 3 == 1 ? 1 : 0); };
      auto addr_of = [&](int t) { return 2 * slot_of(t) + (t % 3 == 2 ? 1 : 0); };
      const int op0 = (int)ops.size();
      for (int t = 0; t < taps; t += 2) {
        if (t + 1 >= taps) {
          ops.push_back(SchedOp{slot_of(t), 2 * E, t, 0, -1, 0});
        } else {
          const int lo = addr_of(t) < addr_of(t + 1) ? t : t + 1, hi = lo == t ? t + 1 : t;
          ops.push_back(SchedOp{slot_of(lo), 2 * E, lo, slot_of(hi), 2 * E, hi});
        }
      }
      push_kb(2 * E, 1, 0, 6, op0);
    }
  } else {
    const int pairs = (cin_chunks + 1) / 2;
    for (int t = 0; t < taps; ++t) {
      for (int g = 0; g * d.cp < pairs; ++g) {
        const int prs = std::min(d.cp, pairs - g * d.cp), op0 = (int)ops.size(), c0 = 2 * g * d.cp;
        const int loaded = std::min(2 * prs, cin_chunks - c0);
        for (int i = 0; i < prs; ++i)
          ops.push_back(2 * i + 1 < loaded ? SchedOp{2 * i, c0 + 2 * i, t, 2 * i + 1, c0 + 2 * i + 1, t}
                                           : SchedOp{2 * i, c0 + 2 * i, t, 0, -1, 0});
        push_kb(c0, loaded, t, 1, op0);
      }
    }
  }
  return 0;
}

struct ConvLaunch {
  ConvParams p;
  dim3 grid;
  int smem;
  int mode, stages, threads;
  bool pdl = true;  // programmatic dependent launch after the previous kernel of its stream
};

// sm_budget: the SMs the launch may spread over (a branch group's share), 0 for all of them.
int build_conv(const ixb_conv_desc& d, uint8_t* arena, uint64_t arena_bytes, int batch, ConvLaunch& L,
               std::string& err, int sm_budget = 0) {
  char buf[256];
  auto bad = [&](const char* m) {
    err = m;
    return -1;
  };
  if (batch < 1) return bad("batch < 1");
  if (d.mode < IXB_MODE_WINDOW || d.mode > IXB_MODE_IM2COL) return bad("unknown conv mode");
  if (d.s2d_in) {
    // a stride-2 3x3 conv over the space-to-depth view: a stride-1 2x2 conv, output size = view size
    if (d.mode != IXB_MODE_WINDOW || d.k != 2 || d.stride != 1 || (d.s2d_in == 1 ? d.cin % 64 : d.cin != 16) ||
        d.s2d_in < 1 || d.s2d_in > 2)
      return bad("a space-to-depth input needs a WINDOW 2x2 stride-1 conv over 4 x whole chunks (the image: one chunk)");
    if (d.out_h != d.in_h || d.out_w != d.in_w) return bad("a space-to-depth conv keeps the view's size");
  } else {
    if (!(d.k == 1 || d.k == 3) || !(d.stride == 1 || d.stride == 2)) return bad("k must be 1 or 3, stride 1 or 2");
    const int pk = d.k / 2;
    if (d.out_h != (d.in_h + 2 * pk - d.k) / d.stride + 1 || d.out_w != (d.in_w + 2 * pk - d.k) / d.stride + 1)
      return bad("output size does not follow from input size, k and stride");
  }
  if (d.nseg < 1 || d.nseg > IXB_MAX_SEGS) return bad("1..4 input segments");
  // window reach before a pixel: one row and one column for 3x3 and the 2x2 space-to-depth taps
  const int pad = d.s2d_in ? 1 : d.k / 2;
  if (d.cout % 16 || d.n_tile % 16 || d.n_tile < 16 || d.n_tile > 256 || d.cout % d.n_tile)
    return bad("cout and n_tile must be multiples of 16, n_tile <= 256 dividing cout");
  if (!(d.cp == 1 || d.cp == 2 || d.cp == 4)) return bad("cp must be 1, 2 or 4");
  // SRS shifts: the float path of the epilogue is exact for s <= 16 (and for s < 0, a left shift);
  // larger s first reduce the accumulator exactly by s - 16 (a sticky bit keeps the rounding).
  if (d.shift < -31 || d.shift > 47) return bad("shift outside [-31, 47]");
  ConvParams& p = L.p;
  memset(&p, 0, sizeof p);
  p.mode = d.mode;
  p.k = d.k;
  p.stride = d.stride;
  p.pad = pad;
  p.H = d.in_h;
  p.W = d.in_w;
  p.Ho = d.out_h;
  p.Wo = d.out_w;
  // STEM and IM2COL compute one spare output column per row so that a one-row descriptor shift
  // (the neighbouring tap) never crosses into the next output row
  p.Wm = (d.mode == IXB_MODE_STEM || d.mode == IXB_MODE_IM2COL) ? d.out_w + 1 : d.out_w;
  p.batch = batch;
  p.cp = d.cp;
  p.n_tile = d.n_tile;
  p.cout = d.cout;
  p.nseg = d.nseg;
  int cin = 0;
  int chunk = 0;
  for (int i = 0; i < d.nseg; ++i) {
    const ixb_segment& s = d.seg[i];
    const bool image = d.mode == IXB_MODE_STEM;
    if (check_seg(s, batch, arena_bytes, image, "conv input", err)) return -1;
    const int sh = s.up2 ? 2 * s.height : s.height, sw = s.up2 ? 2 * s.width : s.width;
    if (sh != d.in_h || sw != d.in_w) return bad("input segment size differs from the conv input size");
    if (s.up2 && (d.mode != IXB_MODE_GATHER || d.k != 1 || d.stride != 1))
      return bad("an up2 input needs GATHER mode and a 1x1 stride-1 conv");
    p.seg[i] = seg_dev(s, arena, chunk);
    chunk += image ? 1 : p.seg[i].chunks;
    cin += s.channels;
  }
  if (cin != d.cin) return bad("segment channels do not add up to cin");
  switch (d.mode) {
    case IXB_MODE_WINDOW:
      if (d.stride != 1) return bad("WINDOW mode is stride 1");
      break;
    case IXB_MODE_STEM:
      if (d.k != 3 || d.stride != 2 || d.nseg != 1 || d.cin != 3 || d.in_h % 2 || d.in_w % 2)
        return bad("STEM mode is a 3x3 stride-2 conv of the 3-channel image with an even size");
      break;
    case IXB_MODE_IM2COL:
      if (d.k != 3 || d.stride != 2 || d.nseg != 1 || d.in_h % 2 || d.in_w % 2 || !p.seg[0].plane_images)
        return bad("IM2COL mode is a 3x3 stride-2 conv of one view with whole-image plane strides and an even size");
      if (d.in_w + 2 > 256 * 16 || d.in_h + 2 > 65535) return bad("IM2COL input too large");
      break;
    default:
      if (d.k != 1 || d.stride != 1) return bad("GATHER mode is a 1x1 stride-1 conv");
      break;
  }
  p.cin_chunks = chunk;
  if (d.mode == IXB_MODE_WINDOW) {
    p.win_origin = pad * (d.in_w + 2) + pad;
    p.m_total = (int)std::min<long long>(0x7fffffffLL, (long long)batch * (d.in_h + 2) * (d.in_w + 2));
  } else {
    p.win_origin = 0;
    p.m_total = (int)std::min<long long>(0x7fffffffLL, (long long)batch * d.out_h * p.Wm);
  }
  if ((long long)batch * (d.in_h + 2) * (d.in_w + 4) >= 0x7fff0000LL)
    return bad("more pixels than 32-bit pixel indices cover");
  std::vector<SchedKB> kbs;
  std::vector<SchedOp> ops;
  build_schedule(d, chunk, kbs, ops);
  if ((int)kbs.size() > kMaxKBlocks) return bad("too many K-blocks for the schedule table");
  p.kblocks = (int)kbs.size();
  int slots = 0, b_stage_max = 0;
  for (const SchedKB& k : kbs) {
    slots = std::max(slots, k.nchunks * k.ntaps);
    b_stage_max = std::max(b_stage_max, k.b_bytes);
  }
  const int b_total = kbs.back().b_off + kbs.back().b_bytes;
  const long long ntiles = d.cout / d.n_tile;
  if ((unsigned long long)ntiles * b_total != d.w_bytes) {
    snprintf(buf, sizeof buf, "packed weights are %llu bytes, the schedule needs %llu",
             (unsigned long long)d.w_bytes, (unsigned long long)(ntiles * b_total));
    err = buf;
    return -1;
  }
  if (d.w_offset % 16 || d.w_offset + d.w_bytes > arena_bytes) return bad("weights outside the arena or misaligned");
  if (d.bias_offset % 16 || d.bias_offset + 4ull * d.cout > arena_bytes) return bad("bias outside the arena");
  if (d.lut_offset + 256 > arena_bytes) return bad("activation table outside the arena");
  // Tile of MT blocks of 128 pixels: the largest MT that keeps two accumulators within TMEM
  // (2 * MT * n_tile <= 512 columns) and still leaves two tiles per SM to spread.
  const int sms = sm_budget > 0 ? std::min(sm_budget, sm_count()) : sm_count();
  int mt = 1;
  // WINDOW convs may take 8 or 16 blocks (up to 2048 rows; the planner's plane guards cover that
  // reach): for the 16-channel stem this took 85 to 69 us. IM2COL/STEM loads carry at most 1024
  // rows with their halo and the GATHER row tables hold 512, so those stay at 4.
  // A WINDOW tile's last window reaches m_tiles * tile_rows + win_origin pixels into the planes: a
  // candidate whose reach passes the smallest input guard is skipped, so views planned with smaller
  // guards (1024 + 2 (W + 3) + 64 pixels) still build, with smaller tiles.
  int min_guard = 0x7fffffff;
  for (int i = 0; i < d.nseg; ++i) min_guard = std::min(min_guard, d.seg[i].guard);
  const long long plane_px = (long long)batch * (d.in_h + 2) * (d.in_w + 2);
  for (int cand : {16, 8, 4, 2}) {
    if (cand >= 8 && d.mode != IXB_MODE_WINDOW) continue;
    const long long tiles = (p.m_total + 128LL * cand - 1) / (128LL * cand);
    if (d.mode == IXB_MODE_WINDOW && tiles * 128LL * cand + p.win_origin > plane_px + min_guard) continue;
    if (cand * d.n_tile <= 256 && tiles * ntiles >= 2LL * sms) {
      mt = cand;
      break;
    }
  }
  p.b_block_bytes = b_stage_max;
  // barriers, bias, per-chunk table (WINDOW: plane addresses, GATHER: GatherChunk), gather row tables
  const int ctab_entry = d.mode == IXB_MODE_GATHER ? (int)sizeof(GatherChunk) : 8;
  const int extra = 512 + 1024 + ctab_entry * chunk + 16 + (d.mode == IXB_MODE_GATHER ? 2 * 512 * 16 : 0);
  const int budget = kConvDynSmem - 1024 - extra;
  for (;; mt /= 2) {
    p.mt = mt;
    p.tile_rows = 128 * mt;
    // WINDOW: taps reach win_origin pixels back and (3x3) as far ahead; the 2x2 taps only back
    p.rowsA = (d.mode == IXB_MODE_WINDOW) ? p.tile_rows + (d.s2d_in ? 1 : 2) * p.win_origin
              : ((d.mode == IXB_MODE_STEM || d.mode == IXB_MODE_IM2COL) ? p.tile_rows + 8 : p.tile_rows);
    // 16 spare bytes: a single-tap MMA's unused second K-half reads one row past its slot
    p.a_stage_bytes = slots * p.rowsA * 16 + 16;
    p.b_resident = b_total <= budget / 2 ? 1 : 0;
    const int res_bytes = p.b_resident ? round_up(b_total, 1024) : 0;
    p.stage_bytes = round_up(p.a_stage_bytes + (p.b_resident ? 0 : b_stage_max), 1024);
    const int S = std::min(6, (budget - res_bytes) / p.stage_bytes);
    if (S >= 2) {
      p.stages = S;
      p.a_off = res_bytes;
      break;
    }
    if (mt == 1) return bad("a pipeline stage does not fit shared memory");
  }
  p.m_tiles = (int)((p.m_total + p.tile_rows - 1) / p.tile_rows);
  p.tbl_off = p.a_off + p.stages * p.stage_bytes;
  p.bar_off = p.tbl_off + (d.mode == IXB_MODE_GATHER ? 2 * p.tile_rows * 16 : 0);
  p.bias_off = p.bar_off + 512;
  if ((d.mode == IXB_MODE_IM2COL || d.mode == IXB_MODE_STEM) && p.rowsA > 1024)
    return bad("an im2col load carries at most 1024 pixels");
  // Warps: 16 epilogue + 1 producer + 3 MMA warps (GATHER: 8 + 4 producer warps + 4); the issuers
  // split each K-block's MMAs between them.
  p.ew = d.mode == IXB_MODE_GATHER ? 8 : 16;
  p.issuers = mma_warps(p.ew);
  p.w_ntile_stride = (long long)b_total;
  p.wpack = arena + d.w_offset;
  p.bias = reinterpret_cast<const int32_t*>(arena + d.bias_offset);
  p.lut = reinterpret_cast<const int8_t*>(arena + d.lut_offset);
  p.shift = std::min(d.shift, 16);
  p.pre_shift = std::max(d.shift - 16, 0);
  p.fd_P = make_fastdiv((uint32_t)((d.in_h + 2) * (d.in_w + 2)));
  p.fd_W2 = make_fastdiv((uint32_t)(d.in_w + 2));
  p.fd_hw = make_fastdiv((uint32_t)(d.out_h * p.Wm));
  p.fd_Wo = make_fastdiv((uint32_t)p.Wm);
  p.acc_cols = p.mt * d.n_tile;
  // as many accumulators as TMEM's 512 columns hold, 2 to 8: the spare ones let the MMAs run
  // ahead of the epilogue and absorb the jitter between the two
  p.nacc = std::max(2, std::min(kMaxAcc, 512 / p.acc_cols));
  if (p.nacc * p.acc_cols > 512) return bad("the accumulators do not fit TMEM");
  int cols = 32;
  while (cols < p.nacc * p.acc_cols) cols *= 2;
  p.tmem_cols = cols;
  if ((2 * p.stages + 2 * p.nacc + 1) * 8 + 4 > 512) return bad("too many pipeline stages");
  p.idesc = umma_idesc_s8(kBlockM, d.n_tile);
  {
    // kernel op table: A start / LBO from (slot, tap) and the geometry, deduplicated per K-block
    auto shift_of = [&](int t) {
      if (d.mode == IXB_MODE_WINDOW) return (t / d.k) * (d.in_w + 2) + (t % d.k);
      if (d.mode == IXB_MODE_STEM) return t & 1;
      return d.mode == IXB_MODE_IM2COL && t % 3 == 2 ? 1 : 0;
    };
    std::vector<uint32_t> ta;
    std::vector<uint16_t> tb;
    for (size_t i = 0; i < kbs.size(); ++i) {
      const SchedKB& k = kbs[i];
      std::vector<uint32_t> ka;
      std::vector<uint16_t> kbv;
      for (int o = 0; o < k.nops; ++o) {
        const SchedOp& op = ops[k.op0 + o];
        const int a_start = op.slot0 * p.rowsA + shift_of(op.tap0);
        int lbo = 1;
        if (op.chunk1 >= 0) lbo = op.slot1 * p.rowsA + shift_of(op.tap1) - a_start;
        if (lbo <= 0 || lbo >= (1 << 14) || a_start >= (1 << 14)) return bad("MMA operand offsets out of range");
        // rows read: a_start .. a_start + tile_rows - 1 (+ lbo for the second K-half), within the A region + 16
        if ((long long)(a_start + lbo + p.tile_rows) * 16 > p.a_stage_bytes)
          return bad("an MMA operand reads past its stage");
        ka.push_back((uint32_t)a_start | ((uint32_t)lbo << 16));
        kbv.push_back((uint16_t)(o * d.n_tile * 32 / 16));
      }
      int found = -1;
      for (size_t st = 0; st + ka.size() <= ta.size() && found < 0; ++st) {
        bool eq = true;
        for (size_t j = 0; j < ka.size() && eq; ++j) eq = ta[st + j] == ka[j] && tb[st + j] == kbv[j];
        if (eq) found = (int)st;
      }
      if (found < 0) {
        found = (int)ta.size();
        ta.insert(ta.end(), ka.begin(), ka.end());
        tb.insert(tb.end(), kbv.begin(), kbv.end());
      }
      if ((int)ta.size() > kMaxOps) return bad("too many MMAs for the op table");
      KBlockDev& kd = p.kb[i];
      kd.b_off = k.b_off;
      kd.b_bytes = k.b_bytes;
      kd.op0 = (int16_t)found;
      kd.nops = (int16_t)k.nops;
      kd.chunk0 = (int16_t)k.chunk0;
      kd.nchunks = (int16_t)k.nchunks;
      kd.tap0 = (int16_t)k.tap0;
      kd.ntaps = (int16_t)k.ntaps;
    }
    for (size_t i = 0; i < ta.size(); ++i) {
      p.op_a[i] = ta[i];
      p.op_b[i] = tb[i];
    }
  }
  p.has_res = d.has_residual;
  if (d.has_residual) {
    if (d.mode != IXB_MODE_WINDOW) return bad("a residual needs WINDOW mode");
    if (check_seg(d.residual, batch, arena_bytes, false, "residual", err)) return -1;
    if (d.residual.height != d.out_h || d.residual.width != d.out_w || d.residual.channels != d.cout ||
        d.residual.up2)
      return bad("residual view must match the output");
    // (t2 << lsh_m) + (r << lsh_r) stays below 2^24 in magnitude, where the float rounding is exact
    if (d.res_lsh_main < 0 || d.res_lsh_main > 16 || d.res_lsh_res < 0 || d.res_lsh_res > 16 ||
        d.res_shift < 0 || d.res_shift > 31)
      return bad("residual shifts outside [0, 16] (left) or [0, 31] (rounding)");
    p.res = seg_dev(d.residual, arena, 0);
    p.res_lsh_m = d.res_lsh_main;
    p.res_lsh_r = d.res_lsh_res;
    p.res_shift = d.res_shift;
  }
  p.out_nchw = d.out_nchw;
  if (d.out2_kind < IXB_OUT2_NONE || d.out2_kind > IXB_OUT2_S2D_ONLY) return bad("unknown out2_kind");
  if (d.out_nchw && d.out2_kind) return bad("an NCHW head has no second output");
  if (!d.out_nchw) {
    if (d.out2_kind != IXB_OUT2_S2D_ONLY) {  // the space-to-depth-only output leaves `out` unused
      if (check_seg(d.out, batch, arena_bytes, false, "conv output", err)) return -1;
      if (d.out.height != d.out_h || d.out.width != d.out_w || d.out.channels != d.cout || d.out.up2)
        return bad("output view must be out_h x out_w x cout");
      p.out = seg_dev(d.out, arena, 0);
    }
  } else {
    const unsigned long long plane = (unsigned long long)d.out_h * d.out_w;
    const int ech = d.egress_channels ? d.egress_channels : d.cout;
    if (ech < 0 || ech > d.cout || d.cout - ech >= 16) return bad("egress channels must lie in (cout - 16, cout]");
    if (d.egress_image_bytes < plane * ech ||
        d.egress_offset + (unsigned long long)(batch - 1) * d.egress_image_bytes + plane * ech > arena_bytes)
      return bad("head egress outside the arena");
    p.egress_ch = ech;
    p.egress = reinterpret_cast<int8_t*>(arena + d.egress_offset);
    p.egress_img = (long long)d.egress_image_bytes;
  }
  p.out2_kind = d.out2_kind;
  if (d.out2_kind) {
    if (check_seg(d.out2, batch, arena_bytes, false, "conv second output", err)) return -1;
    if (d.out2.up2) return bad("the second output view is not an up2 view");
    if (d.out2_kind == IXB_OUT2_UP2) {
      if (d.out2.height != 2 * d.out_h || d.out2.width != 2 * d.out_w || d.out2.channels != d.cout)
        return bad("the upsampled output view must be 2 out_h x 2 out_w x cout");
    } else {
      if (d.out_h % 2 || d.out_w % 2 || d.out2.height != d.out_h / 2 || d.out2.width != d.out_w / 2 ||
          d.out2.channels != 4 * d.cout)
        return bad("the space-to-depth output view must be out_h/2 x out_w/2 x 4 cout (even sizes)");
    }
    p.out2 = seg_dev(d.out2, arena, 0);
  }
  if (d.mode == IXB_MODE_WINDOW) {
    auto same = [&](const ixb_segment& s) { return s.height == d.in_h && s.width == d.in_w; };
    for (int i = 0; i < d.nseg; ++i)
      if (!same(d.seg[i])) return bad("WINDOW views must share the input geometry");
    if (!d.out_nchw && d.out2_kind != IXB_OUT2_S2D_ONLY && !same(d.out))
      return bad("WINDOW output must share the input geometry");
    // every window copy stays inside the planes' zero guards
    for (int i = 0; i < d.nseg; ++i) {
      const long long end = (long long)p.m_tiles * p.tile_rows + p.win_origin;
      if (p.win_origin > d.seg[i].guard || end > (long long)batch * (d.in_h + 2) * (d.in_w + 2) + d.seg[i].guard)
        return bad("input plane guards are smaller than the window over-reach");
    }
  }
  p.ctab_off = round_up(p.bias_off + 4 * d.n_tile, 16);
  const int smem = p.ctab_off + ctab_entry * p.cin_chunks + 1024;
  if (smem > kConvDynSmem) return bad("shared memory plan exceeds the limit");
  const long long gm = std::max<long long>(1, std::min<long long>(p.m_tiles, ((long long)sms + ntiles - 1) / ntiles));
  L.grid = dim3((unsigned)gm, (unsigned)ntiles, 1);
  L.smem = smem;
  L.mode = d.mode;
  L.stages = p.stages;
  L.threads = conv_threads(d.mode, p.ew);
  return 0;
}

// The TMA im2col map of an IM2COL or STEM conv (needs the driver; done at launch, not in the checks).
// IM2COL: the view's chunk planes as one 4-D tensor {16 B, W+2, H+2, images}: chunk c of image n is
// image c * plane_images + n; corners 0 / -2 and element strides 2 walk the 3x3 stride-2 windows.
// STEM: the image plane as 16-byte pixel pairs {16 B, (W+4)/2, H+2, batch}: element strides (1, 2).
int encode_im2col(ConvLaunch& L, const ixb_conv_desc& d, uint8_t* arena, int batch, std::string& err) {
  static PFN_cuTensorMapEncodeIm2col_v12000 enc = nullptr;
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", (void**)&enc, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !enc) {
      enc = nullptr;
      err = "cuTensorMapEncodeIm2col is not available";
      return -1;
    }
  }
  ConvParams& p = L.p;
  cuuint64_t dims[4], strides[3];
  cuuint32_t es[4];
  void* base;
  if (d.mode == IXB_MODE_IM2COL) {
    const SegDev& s = p.seg[0];
    base = const_cast<int8_t*>(s.base);
    dims[0] = 16;
    dims[1] = (cuuint64_t)(s.W + 2);
    dims[2] = (cuuint64_t)(s.H + 2);
    dims[3] = (cuuint64_t)((long long)(s.chunks - 1) * s.plane_images + batch);
    strides[0] = 16;
    strides[1] = (cuuint64_t)(s.W + 2) * 16;
    strides[2] = (cuuint64_t)s.P * 16;
    es[0] = 1; es[1] = 2; es[2] = 2; es[3] = 1;
  } else {
    const ixb_segment& s = d.seg[0];
    base = arena + s.offset;
    dims[0] = 16;
    dims[1] = (cuuint64_t)((s.width + 4) / 2);
    dims[2] = (cuuint64_t)(s.height + 2);
    dims[3] = (cuuint64_t)batch;
    strides[0] = 16;
    strides[1] = (cuuint64_t)(s.width + 4) * 8;
    strides[2] = (cuuint64_t)(s.height + 2) * (s.width + 4) * 8;
    es[0] = 1; es[1] = 1; es[2] = 2; es[3] = 1;
  }
  // corners (W, H): Ho rows of stride-2 windows, and Wo + 1 window positions per row (a spare output
  // column, so the one-row shift to the neighbouring tap stays within the row); tile + 8 rows a load
  int lower[2] = {0, 0}, upper[2] = {-1, -2};
  CUresult r = enc(&p.tmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, dims, strides, lower, upper, 16,
                   (cuuint32_t)p.rowsA, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeIm2col failed (" + std::to_string((int)r) + ")";
    return -1;
  }
  return 0;
}

// Kernels of a network step are launched with programmatic stream serialization: each may begin
// its setup while the previous kernel drains (the kernels wait for the previous grid before any
// activation access). IXB_PDL=0 turns it off.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("IXB_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t st, bool pdl,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <int MODE, int EW>
int launch_conv_m(const ConvLaunch& L, cudaStream_t st) {
  if (int r = ensure_smem_limit(conv_kernel<MODE, EW>, kConvDynSmem)) return r;
  IXB_CUDA(launch_dependent(conv_kernel<MODE, EW>, L.grid, dim3(conv_threads(MODE, EW)), L.smem, st, L.pdl, L.p));
  return 0;
}

int launch_conv(const ConvLaunch& L, cudaStream_t st) {
  switch (L.mode) {
    case IXB_MODE_WINDOW: return launch_conv_m<IXB_MODE_WINDOW, 16>(L, st);
    case IXB_MODE_GATHER: return launch_conv_m<IXB_MODE_GATHER, 8>(L, st);
    case IXB_MODE_IM2COL: return launch_conv_m<IXB_MODE_IM2COL, 16>(L, st);
    default: return launch_conv_m<IXB_MODE_STEM, 16>(L, st);
  }
}

// Host checks, then (for im2col modes) the tensor map: everything a launch needs.
int prepare_conv(const ixb_conv_desc& d, uint8_t* arena, uint64_t arena_bytes, int batch, ConvLaunch& L,
                 std::string& err, int sm_budget = 0) {
  if (build_conv(d, arena, arena_bytes, batch, L, err, sm_budget)) return -1;
  if (d.mode == IXB_MODE_IM2COL || d.mode == IXB_MODE_STEM) return encode_im2col(L, d, arena, batch, err);
  return 0;
}

struct PoolLaunch {
  PoolParams p;
  dim3 grid;
  int smem;
};

int build_pool(const ixb_pool_desc& d, uint8_t* arena, uint64_t arena_bytes, int batch, PoolLaunch& L,
               std::string& err) {
  memset(&L.p, 0, sizeof L.p);
  if (check_seg(d.in, batch, arena_bytes, false, "pool input", err)) return -1;
  if (d.in.up2) {
    err = "pool input cannot be an up2 view";
    return -1;
  }
  for (int k = 0; k < 3; ++k) {
    if (check_seg(d.out[k], batch, arena_bytes, false, "pool output", err)) return -1;
    if (d.out[k].height != d.in.height || d.out[k].width != d.in.width || d.out[k].channels != d.in.channels ||
        d.out[k].up2) {
      err = "pool outputs must match the input";
      return -1;
    }
  }
  const int n = d.in.height * d.in.width;
  L.smem = 3 * n * 16;
  if (L.smem > kSmemLimit) {
    err = "pool plane does not fit shared memory";
    return -1;
  }
  L.p.in = seg_dev(d.in, arena, 0);
  for (int k = 0; k < 3; ++k) L.p.out[k] = seg_dev(d.out[k], arena, 0);
  L.p.H = d.in.height;
  L.p.W = d.in.width;
  L.p.chunks = d.in.channels / 16;
  if (d.in.height * d.in.width * 16 * 3 > kSmemLimit) {
    err = "pool plane does not fit shared memory";
    return -1;
  }
  L.grid = dim3(L.p.chunks, batch, 1);
  return 0;
}

int launch_pool(const PoolLaunch& L, cudaStream_t st) {
  if (int r = ensure_smem_limit(sppf_kernel, kSmemLimit)) return r;
  if (int r = ensure_smem_limit(sppf_pixel_kernel, kSmemLimit)) return r;
  const int n = L.p.H * L.p.W;
  if (n <= 1024)  // one thread per pixel
    IXB_CUDA(launch_dependent(sppf_pixel_kernel, L.grid, dim3((unsigned)((n + 31) / 32 * 32)), L.smem, st, true, L.p));
  else
    IXB_CUDA(launch_dependent(sppf_kernel, L.grid, dim3(256), L.smem, st, true, L.p));
  return 0;
}

int launch_quantize(const uint8_t* images, const int8_t* lut, int batch, int h, int w, int8_t* out,
                    cudaStream_t st) {
  if (w % 4) return fail(IXB_ERR_INVALID, "image width must be a multiple of 4");
  const long long items = (long long)batch * h * (w / 2 + 1);
  if (items >= (1LL << 31)) return fail(IXB_ERR_INVALID, "too many pixels for one ingress launch");
  const int blocks = (int)std::min<long long>((items + 255) / 256, 148LL * 16);
  quantize_images_kernel<<<blocks, 256, 0, st>>>(images, lut, batch, h, w, make_fastdiv((uint32_t)(w / 2 + 1)),
                                                 make_fastdiv((uint32_t)h), out);
  IXB_CUDA(cudaGetLastError());
  return 0;
}

// The image's space-to-depth view (ixb_plan.input_s2d): from the uint8 images (the ingress), or
// from the 8-byte-pixel store `in8` (after a letterbox). `view` is the plan's input_s2d_view.
int launch_ingress_s2d(const uint8_t* images, const int8_t* in8, const int8_t* lut, int batch, int h, int w,
                       uint8_t* arena, const ixb_segment& view, cudaStream_t st) {
  if (h % 2 || w % 4) return fail(IXB_ERR_INVALID, "the space-to-depth ingress needs even height, width % 4 == 0");
  const long long items = (long long)batch * (h / 2) * (w / 2);  // view pixels
  if (items >= (1LL << 31)) return fail(IXB_ERR_INVALID, "too many pixels for one ingress launch");
  const int W2 = w / 2 + 2, P2 = (h / 2 + 2) * W2;
  int8_t* out = reinterpret_cast<int8_t*>(arena + view.offset);
  const FastDiv fh = make_fastdiv((uint32_t)(h / 2));
  if (images) {  // one thread per pair of view pixels
    const int blocks = (int)std::min<long long>((items / 2 + 255) / 256, 148LL * 16);
    quantize_images_s2d_kernel<<<blocks, 256, 0, st>>>(images, lut, batch, h, w, make_fastdiv((uint32_t)(w / 4)),
                                                       fh, P2, W2, out);
  } else {
    const int blocks = (int)std::min<long long>((items + 255) / 256, 148LL * 16);
    repack_s2d_kernel<<<blocks, 256, 0, st>>>(in8, batch, h, w, make_fastdiv((uint32_t)(w / 2)), fh, P2, W2, out);
  }
  IXB_CUDA(cudaGetLastError());
  return 0;
}

// ---------------------------------------------------------------- int8 GEMM
PFN_cuTensorMapEncodeTiled_v12000 tiled_encoder(std::string& err) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&enc, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !enc) {
      enc = nullptr;
      err = "cuTensorMapEncodeTiled is not available";
    }
  }
  return enc;
}

// Tensor map of an int8 [rows][K] K-major matrix: boxes of 128 bytes of K by box_rows rows,
// 128-byte swizzled (the UMMA K-major SW128 layout).
int encode_kmajor(CUtensorMap* map, const void* base, long long rows, int K, int box_rows, std::string& err) {
  auto enc = tiled_encoder(err);
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {(cuuint32_t)kGemmBK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return -1;
  }
  return 0;
}

struct GemmLaunch {
  GemmParams p;
  int grid, smem;
};

// Tile shape, pipeline depth and grid for an M x N x K int8 GEMM. The accumulator of a tile is
// MT blocks of 128 rows by BN columns; two of them (2 * MT * BN <= 512 TMEM columns) let the
// epilogue of one tile overlap the next. MT grows only while the tiles still cover every SM.
int plan_gemm(GemmLaunch& L, int M, int N, int K, std::string& err, int bsrc = GEMM_B_TMA) {
  if (M < 1 || N < 16 || N % 16 || K < 16 || K % 16) {
    err = "GEMM shape needs M >= 1, N and K multiples of 16";
    return -1;
  }
  if (bsrc == GEMM_B_W4 && K % kW4Group) {
    err = "W4A8 needs K a multiple of the 128-value group";
    return -1;
  }
  if (K > 65536) {
    err = "K above 65536 could overflow the int32 accumulator";
    return -1;
  }
  GemmParams& p = L.p;
  memset(&p, 0, sizeof p);  // every pointer a variant does not use stays null
  p.M = M;
  p.N = N;
  p.K = K;
  const int sms = sm_count();
  if (bsrc == GEMM_B_W4) {
    // The tile (MT blocks of 128 rows x BN columns) minimising (waves of tiles over the SMs) x
    // (a K-block's time: the slower of its MMAs, 4 x MT of ~max(BN / 2, 32 + BN / 4) cycles with the
    // operands' shared-memory reads bounding narrow ones, and the unpack of BN x 128 int4 values,
    // ~2.5 BN instructions per unpacking warp at ~0.5 per cycle with 4 warps, halved with 8).
    // Two accumulators must fit TMEM, or, when every CTA has at most one tile, one of up to 512
    // columns (MT x BN: the unpacked B tile then serves four 128-row blocks). On a tie the larger
    // tile wins: fewer tiles unpack each weight tile fewer times.
    double best = 1e300;
    const int mt_max = (int)std::min<long long>(4, (M + 127) / 128);
    for (int mt : {1, 2, 4}) {
      if (mt > mt_max && mt != 1) continue;
      for (int bn = 16; bn <= std::min(std::min(512 / mt, 256), round_up(N, 16)); bn += 16) {
        const long long tiles = ((M + 128LL * mt - 1) / (128LL * mt)) * ((N + bn - 1) / bn);
        const long long waves = (tiles + sms - 1) / sms;
        if (mt * bn > 256 && waves > 1) continue;
        const double mma = 4.0 * mt * std::max(bn / 2.0, 32.0 + bn / 4.0);
        const double unpack = 5.0 * bn * 4.0 / kW4Warps;
        const double cost = (double)waves * std::max(mma, unpack);
        if (cost < best - 1e-9 || (cost < best + 1e-9 && mt * bn > p.mt * p.bn)) {
          best = cost;
          p.mt = mt;
          p.bn = bn;
        }
      }
    }
  } else {
    p.bn = N <= 256 ? N : (N % 256 == 0 ? 256 : (N % 128 == 0 ? 128 : 256));
    p.mt = 1;
    const int nt = (N + p.bn - 1) / p.bn;
    for (int cand : {4, 2}) {
      const long long tiles = ((M + 128LL * cand - 1) / (128LL * cand)) * nt;
      // two accumulators of MT x BN columns, or (BN = 256) one 256 x 256 tile filling TMEM: twice
      // the MMA work per operand byte, which the large square GEMMs need (L2 -> shared traffic)
      if ((cand * p.bn <= 256 || (p.bn == 256 && cand == 2)) && tiles >= sms) {
        p.mt = cand;
        break;
      }
    }
  }
  p.n_tiles = (N + p.bn - 1) / p.bn;
  p.m_tiles = (int)((M + 128LL * p.mt - 1) / (128LL * p.mt));
  p.kblocks = (K + kGemmBK - 1) / kGemmBK;
  p.stage_bytes = p.mt * kGemmABlock + p.bn * kGemmBK;
  p.stage_tx = p.stage_bytes;
  if (bsrc == GEMM_B_W4) {  // the packed int4 tile lands after the unpacked B operand
    p.raw_off = p.stage_bytes;
    p.stage_bytes = round_up(p.stage_bytes + p.bn * (kGemmBK / 2), 1024);
    p.stage_tx = p.mt * kGemmABlock + p.bn * (kGemmBK / 2);
  }
  // W4A8: two tiles' group exponents in shared memory (the producer copies the next tile's while
  // the current one unpacks) when one takes at most 16 KB
  const int eg_tile = bsrc == GEMM_B_W4 ? round_up(p.bn * (K / kW4Group), 128) : 0;
  const int eg_bytes = (eg_tile > 0 && eg_tile <= 16 * 1024) ? 2 * eg_tile : 0;
  const int budget = kSmemLimit - 1024 - kGemmBarBytes - eg_bytes;
  p.stages = std::min(kGemmMaxStages, budget / p.stage_bytes);
  if (p.stages < 2) {
    err = "two GEMM pipeline stages do not fit shared memory";
    return -1;
  }
  p.eg_off = eg_bytes ? p.stages * p.stage_bytes : -1;
  p.eg_stride = eg_tile;
  p.bar_off = p.stages * p.stage_bytes + eg_bytes;
  p.acc_cols = p.mt * p.bn;
  p.nacc = 2 * p.acc_cols <= 512 ? 2 : 1;  // one accumulator only for a 512-column tile
  int cols = 32;
  while (cols < p.nacc * p.acc_cols) cols *= 2;
  p.tmem_cols = cols;
  p.idesc = umma_idesc_s8(128, p.bn);
  const long long tiles = (long long)p.m_tiles * p.n_tiles;
  if (tiles > 0x7fffffffLL) {
    err = "too many GEMM tiles";
    return -1;
  }
  L.grid = (int)std::min<long long>(tiles, sms);
  L.smem = 1024 + p.bar_off + kGemmBarBytes;
  return 0;
}

// Tensor map of the W4A8 weight image's packed part: uint8 [N][K/2], boxes of 64 bytes (128
// values, one group) by BN rows, no swizzle; rows past N read as zero.
int encode_w4(CUtensorMap* map, const void* base, int N, int K, int box_rows, std::string& err) {
  auto enc = tiled_encoder(err);
  if (!enc) return -1;
  cuuint64_t dims[2] = {(cuuint64_t)(K / 2), (cuuint64_t)N};
  cuuint64_t strides[1] = {(cuuint64_t)(K / 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "cuTensorMapEncodeTiled failed for the W4A8 weights (" + std::to_string((int)r) + ")";
    return -1;
  }
  return 0;
}

template <int BSRC>
int launch_gemm(GemmLaunch& L, cudaStream_t st) {
  if (int r = ensure_smem_limit(gemm_kernel<8, BSRC>, kSmemLimit)) return r;
  gemm_kernel<8, BSRC><<<L.grid, gemm_threads(8, BSRC), L.smem, st>>>(L.p);
  IXB_CUDA(cudaGetLastError());
  return 0;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

int run_i8gemm(const int8_t* a, const int8_t* b, const int32_t* bias, int8_t* out8, int32_t* out32, int M, int N,
               int K, int shift, int kind, void* stream) {
  if (!a || !b || (kind == GEMM_OUT_SRS && (!bias || !out8)) || (kind == GEMM_OUT_I32 && !out32))
    return fail(IXB_ERR_INVALID, "null argument");
  if (!aligned16(a) || !aligned16(b) || (bias && !aligned16(bias)) || (out8 && !aligned16(out8)) ||
      (out32 && !aligned16(out32)))
    return fail(IXB_ERR_INVALID, "GEMM operands must be 16-byte aligned");
  if (kind == GEMM_OUT_SRS && (shift < 0 || shift > 23)) return fail(IXB_ERR_INVALID, "shift outside [0, 23]");
  GemmLaunch L;
  std::string err;
  if (plan_gemm(L, M, N, K, err)) return fail(IXB_ERR_INVALID, err);
  L.p.out_kind = kind;
  L.p.bias = bias;
  L.p.shift = shift;
  L.p.out8 = out8;
  L.p.out32 = out32;
  if (encode_kmajor(&L.p.ta, a, M, K, 128, err) || encode_kmajor(&L.p.tb, b, N, K, L.p.bn, err))
    return fail(IXB_ERR_CUDA, err);
  return launch_gemm<GEMM_B_TMA>(L, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- W4A8
uint64_t w4a8_image_bytes(int K, int N) { return (uint64_t)N * (K / 2) + (uint64_t)N * (K / kW4Group); }

int check_w4a8_shape(int N, int K) {
  if (N < 16 || N % 16 || K < kW4Group || K % kW4Group || K > 65536)
    return fail(IXB_ERR_INVALID, "W4A8 needs N a multiple of 16 and K a multiple of 128, at most 65536");
  return 0;
}

int read_device_error() {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_dev_error, sizeof v);
  if (e != cudaSuccess) return cuda_fail(e, "reading the device error flag");
  if (v) {
    unsigned int z = 0;
    cudaMemcpyToSymbol(g_dev_error, &z, sizeof z);
    if (v == DEV_ERR_BAD_ARGS) return fail(IXB_ERR_INVALID, "a kernel found invalid input values");
    return fail(IXB_ERR_DEVICE, "a kernel's bounded wait gave up (device error flag " + std::to_string(v) + ")");
  }
  return 0;
}

// Arena bytes an access touches: `count` repeats of [start, start + len), `stride` bytes apart.
struct Span {
  unsigned long long start, len, stride;
  int count;
};

Span view_span(const ixb_segment& s, int batch) {
  if (!s.plane_stride)  // the stem's image store: one block of 8-byte pixels
    return {s.offset, (unsigned long long)batch * (s.height + 2) * (s.width + 4) * 8, 0, 1};
  const unsigned long long chunks = (unsigned long long)(s.channels + 15) / 16;
  return {s.offset - (unsigned long long)s.guard * 16 + (unsigned long long)s.chunk_offset * s.plane_stride,
          chunks * s.plane_stride, 0, 1};
}

bool spans_overlap(const Span& a, const Span& b) {
  auto end = [](const Span& s) { return s.start + (s.count > 1 ? (s.count - 1) * s.stride : 0) + s.len; };
  if (a.start >= end(b) || b.start >= end(a)) return false;
  if (a.count > 1 && b.count > 1 && a.stride == b.stride && a.len <= a.stride && b.len <= b.stride) {
    // pieces repeating with one period (heads inside the per-image egress): compare within a period
    const unsigned long long S = a.stride;
    const unsigned long long d = b.start >= a.start ? (b.start - a.start) % S : (S - (a.start - b.start) % S) % S;
    return d < a.len || S - d < b.len;
  }
  return true;  // conservative
}

void conv_spans(const ixb_conv_desc& d, int batch, std::vector<Span>& rd, std::vector<Span>& wr) {
  for (int i = 0; i < d.nseg && i < IXB_MAX_SEGS; ++i) rd.push_back(view_span(d.seg[i], batch));
  if (d.has_residual) rd.push_back(view_span(d.residual, batch));
  if (d.out_nchw) {
    const int ech = d.egress_channels ? d.egress_channels : d.cout;
    wr.push_back({d.egress_offset, (unsigned long long)d.out_h * d.out_w * ech, d.egress_image_bytes, batch});
  } else if (d.out2_kind != IXB_OUT2_S2D_ONLY) {
    wr.push_back(view_span(d.out, batch));
  }
  if (d.out2_kind) wr.push_back(view_span(d.out2, batch));
}

}  // namespace

// The decode kernel's parameters from a caller's descriptor (tables and anchors in device memory).
int prepare_decode(const ixb_decode_desc& d, uint64_t egress_image_bytes, DecodeParams& p) {
  if (d.reg_max != kDfl) return fail(IXB_ERR_UNSUPPORTED, "decode implements the 16-bin DFL head (reg_max 16)");
  if (d.num_classes < 1 || d.num_classes > 256) return fail(IXB_ERR_INVALID, "num_classes outside [1, 256]");
  if (!d.anchor_x || !d.anchor_y || !d.strides) return fail(IXB_ERR_INVALID, "null anchor tables");
  memset(&p, 0, sizeof p);
  int total = 0;
  for (int h = 0; h < 3; ++h) {
    const ixb_decode_head& hd = d.head[h];
    if (!hd.dfl_exp || !hd.sigmoid || hd.anchors < 1 || hd.anchor_offset != total)
      return fail(IXB_ERR_INVALID, "decode head " + std::to_string(h) + ": missing tables or anchors out of order");
    if (!aligned16(hd.dfl_exp))
      return fail(IXB_ERR_INVALID, "decode head " + std::to_string(h) + ": dfl_exp must be 16-byte aligned");
    const uint64_t box_end = hd.box_offset + (uint64_t)4 * kDfl * hd.anchors;
    const uint64_t cls_end = hd.cls_offset + (uint64_t)d.num_classes * hd.anchors;
    if (box_end > egress_image_bytes || cls_end > egress_image_bytes)
      return fail(IXB_ERR_INVALID, "decode head " + std::to_string(h) + " outside the image's egress");
    total += hd.anchors;
    DecodeHeadDev& o = p.head[h];
    o.box_off = (long long)hd.box_offset;
    o.cls_off = (long long)hd.cls_offset;
    o.dfl_exp = hd.dfl_exp;
    o.sigmoid = hd.sigmoid;
    o.sigmoid_low = hd.sigmoid_low;
    // an integer class maximum m survives when m > q_threshold, i.e. m > floor(q_threshold)
    const double qt = hd.q_threshold;
    o.qi = !(qt < 127.0) ? 127 : (qt < -129.0 ? -129 : (int)std::floor(qt));
    o.anchors = hd.anchors;
    o.anchor_offset = hd.anchor_offset;
  }
  if (total > kDecodeMaxAnchors) return fail(IXB_ERR_INVALID, "more than 8400 anchors per image");
  p.egress_image_bytes = (long long)egress_image_bytes;
  p.anchor_x = d.anchor_x;
  p.anchor_y = d.anchor_y;
  p.strides = d.strides;
  p.num_classes = d.num_classes;
  p.conf = d.conf;
  p.iou = d.iou;
  return 0;
}

// One cluster of kDecodeCluster CTAs per image.
int launch_decode(const DecodeParams& p, int batch, cudaStream_t st) {
  if (int r = ensure_smem_limit(yolo_decode_kernel, decode_smem_bytes())) return r;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(batch * kDecodeCluster));
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = (size_t)decode_smem_bytes();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kDecodeCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  IXB_CUDA(cudaLaunchKernelEx(&cfg, yolo_decode_kernel, p));
  return 0;
}

struct ixb_session {
  int device = 0;
  cudaStream_t stream = nullptr;             // compute
  cudaStream_t h2d = nullptr, d2h = nullptr;  // copy streams of submitted runs
  uint8_t* arena = nullptr;
  uint64_t arena_bytes = 0;
  bool own_arena = false;
  ixb_plan plan{};
  std::vector<ixb_conv_desc> convs;
  std::vector<ixb_pool_desc> pools;
  std::vector<ixb_op> ops;
  // branch groups: [begin, end) runs of ops joined by IXB_OP_WITH_PREV (a lone op is a group of one)
  std::vector<std::pair<int, int>> groups;
  cudaStream_t side[IXB_MAX_BRANCHES - 1] = {};
  std::vector<double> conv_cost;  // measured ms of branch-group members run alone (empty: use MACs)
  cudaEvent_t ev_fork = nullptr, ev_join[IXB_MAX_BRANCHES - 1] = {};
  // launches and graphs per (batch, slot): key = batch * kSlots + slot
  static constexpr int kSlots = 1 + IXB_MAX_EXTRA_SLOTS;
  std::map<int, std::vector<ConvLaunch>> conv_launch;
  std::map<int, std::vector<PoolLaunch>> pool_launch;
  std::map<int, cudaGraphExec_t> graphs;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr, ev_done = nullptr;
  bool pending = false;
  float last_ms = 0.f;
  struct Slot {
    uint64_t ticket = 0;
    bool busy = false;
    cudaEvent_t h2d_done = nullptr, t0 = nullptr, t1 = nullptr, d2h_done = nullptr;
    // detection runs (ixb_session_submit_detect / _frames): letterbox and decode events, the
    // batch, the host clock at submit, and where the detections land
    cudaEvent_t pre0 = nullptr, post1 = nullptr;
    bool detections = false, frames = false;
    int batch = 0;
    std::chrono::steady_clock::time_point submitted;
    uint8_t* det_dev = nullptr;   // [counts: max_batch int32][boxes][scores][classes] for this batch
    uint8_t* det_host = nullptr;  // pinned copy of the same
    float* lb_dev = nullptr;      // [max_batch][3] pad_top, pad_left, scale
    float* lb_host = nullptr;     // pinned staging of lb_dev
    uint8_t* frames_dev = nullptr;  // BGR frames of a frames run (grown on demand)
    size_t frames_cap = 0;
  } slots[kSlots];
  // Detection stage (ixb_session_set_detect): decode + NMS after the network.
  bool detect = false;
  ixb_detect_config dcfg{};
  DecodeParams dparams{};
  uint8_t* det_mem = nullptr;   // device memory of every slot's detections and letterbox rows
  uint8_t* det_tables = nullptr;  // the decode tables' score ranks and DFL checks (decode_tables_kernel)
  uint8_t* det_pinned = nullptr;
  std::vector<std::string> class_names;
  ixb_timings last_timings{};
  size_t lb_bytes() const { return ((size_t)plan.max_batch * 12 + 255) / 256 * 256; }
  size_t det_slot_bytes() const {
    const size_t cap = (size_t)dcfg.capacity, B = (size_t)plan.max_batch;
    return ((B * 4 + 255) / 256 * 256 + B * cap * 24 + 255) / 256 * 256 + lb_bytes();
  }
  // The detections of `batch` images, contiguous so one copy brings them back: counts [batch]
  // (padded to 16 bytes), boxes [batch][capacity][4], scores and classes [batch][capacity].
  void det_layout(uint8_t* base, int batch, int32_t** counts, float** boxes, float** scores, int32_t** classes) const {
    const size_t cap = (size_t)dcfg.capacity;
    const size_t c_bytes = ((size_t)batch * 4 + 15) / 16 * 16;
    *counts = reinterpret_cast<int32_t*>(base);
    *boxes = reinterpret_cast<float*>(base + c_bytes);
    *scores = reinterpret_cast<float*>(base + c_bytes + (size_t)batch * cap * 16);
    *classes = reinterpret_cast<int32_t*>(base + c_bytes + (size_t)batch * cap * 20);
  }
  size_t det_bytes(int batch) const { return ((size_t)batch * 4 + 15) / 16 * 16 + (size_t)batch * dcfg.capacity * 24; }
  uint64_t next_ticket = 1;

  int depth() const { return 1 + plan.extra_slots; }
  int slot_of(uint64_t ticket) const { return (int)((ticket - 1) % (uint64_t)depth()); }
  uint64_t images_at(int slot) const { return slot ? plan.extra_images_offset[slot - 1] : plan.images_offset; }
  uint64_t egress_at(int slot) const { return slot ? plan.extra_egress_offset[slot - 1] : plan.egress_offset; }

  int prepare(int batch, int slot = 0) {
    const int key = batch * kSlots + slot;
    if (conv_launch.count(key)) return 0;
    if (slot) {
      // other slots differ only in where the head convs write the egress
      if (int r = prepare(batch, 0)) return r;
      std::vector<ConvLaunch> cl = conv_launch[batch * kSlots];
      const long long delta = (long long)egress_at(slot) - (long long)plan.egress_offset;
      for (ConvLaunch& L : cl)
        if (L.p.out_nchw) L.p.egress += delta;
      conv_launch[key] = std::move(cl);
      pool_launch[key] = pool_launch[batch * kSlots];
      return 0;
    }
    std::vector<ConvLaunch> cl(convs.size());
    std::vector<PoolLaunch> pl(pools.size());
    std::string err;
    // a branch group splits the SMs between its convs in proportion to their device time run alone
    // on the whole GPU (measured when the session is created; MACs until then), at least one CTA
    // per output-channel tile each: members that scale with SMs then take as long as the group's
    // serial time, while latency-bound ones overlap. Members after the first start from the fork,
    // not by programmatic dependent launch.
    std::vector<int> budget(convs.size(), 0);
    std::vector<char> forked(convs.size(), 0);
    const int sms = sm_count();
    for (const auto& g : groups) {
      if (g.second - g.first < 2) continue;
      double total = 0.0;
      std::vector<double> w;
      for (int i = g.first; i < g.second; ++i) {
        const ixb_conv_desc& d = convs[ops[i].index];
        w.push_back(conv_cost.empty() ? (double)d.out_h * d.out_w * d.cin * d.k * d.k * d.cout
                                      : conv_cost[ops[i].index]);
        total += w.back();
      }
      for (int i = g.first; i < g.second; ++i) {
        const ixb_conv_desc& d = convs[ops[i].index];
        const int nt = d.n_tile > 0 ? std::max(1, d.cout / d.n_tile) : 1;
        budget[ops[i].index] = std::max(nt, (int)(sms * w[i - g.first] / (total > 0.0 ? total : 1.0)));
        forked[ops[i].index] = i > g.first;
      }
    }
    for (size_t i = 0; i < convs.size(); ++i) {
      if (prepare_conv(convs[i], arena, arena_bytes, batch, cl[i], err, budget[i]))
        return fail(IXB_ERR_INVALID, "conv " + std::to_string(i) + ": " + err);
      cl[i].pdl = !forked[i];
    }
    for (size_t i = 0; i < pools.size(); ++i)
      if (build_pool(pools[i], arena, arena_bytes, batch, pl[i], err))
        return fail(IXB_ERR_INVALID, "pool " + std::to_string(i) + ": " + err);
    conv_launch[key] = std::move(cl);
    pool_launch[key] = std::move(pl);
    return 0;
  }

  // Device time of each branch-group member run alone on the whole GPU at `batch` images (mean
  // of three launches after one warm-up), for the SM shares; the launches then rebuild.
  int measure_costs(int batch) {
    bool any = false;
    for (const auto& g : groups) any = any || g.second - g.first > 1;
    if (!any) return 0;
    std::vector<double> cost(convs.size(), 0.0);
    cudaEvent_t a = nullptr, b = nullptr;
    IXB_CUDA(cudaEventCreate(&a));
    cudaError_t e = cudaEventCreate(&b);
    int rc = e == cudaSuccess ? 0 : cuda_fail(e, "event creation");
    std::string err;
    for (const auto& g : groups) {
      if (rc || g.second - g.first < 2) continue;
      for (int i = g.first; i < g.second && !rc; ++i) {
        const int idx = ops[i].index;
        ConvLaunch L;
        if (prepare_conv(convs[idx], arena, arena_bytes, batch, L, err)) {
          rc = fail(IXB_ERR_INVALID, "conv " + std::to_string(idx) + ": " + err);
          break;
        }
        L.pdl = false;
        rc = launch_conv(L, stream);
        if (!rc && cudaEventRecord(a, stream) != cudaSuccess) rc = fail(IXB_ERR_CUDA, "event record");
        for (int r = 0; r < 3 && !rc; ++r) rc = launch_conv(L, stream);
        if (!rc && cudaEventRecord(b, stream) != cudaSuccess) rc = fail(IXB_ERR_CUDA, "event record");
        float ms = 0.f;
        if (!rc && cudaEventSynchronize(b) != cudaSuccess) rc = fail(IXB_ERR_CUDA, "event synchronize");
        if (!rc) cudaEventElapsedTime(&ms, a, b);
        cost[idx] = ms / 3.0;
      }
    }
    cudaEventDestroy(a);
    if (b) cudaEventDestroy(b);
    if (rc) return rc;
    conv_cost = std::move(cost);
    conv_launch.clear();
    pool_launch.clear();
    return read_device_error();
  }

  int enqueue_op(int batch, int i, int slot = 0, cudaStream_t st = nullptr) {
    const ixb_op& op = ops[i];
    const int key = batch * kSlots + slot;
    if (!st) st = stream;
    if ((op.kind & 0xFF) == IXB_OP_CONV) return launch_conv(conv_launch[key][op.index], st);
    return launch_pool(pool_launch[key][op.index], st);
  }

  int enqueue_ingress(int batch, int slot = 0) {
    if (plan.input_s2d)
      return launch_ingress_s2d(arena + images_at(slot), nullptr,
                                reinterpret_cast<const int8_t*>(arena + plan.input_lut_offset), batch, plan.img_h,
                                plan.img_w, arena, plan.input_s2d_view, stream);
    return launch_quantize(arena + images_at(slot), reinterpret_cast<const int8_t*>(arena + plan.input_lut_offset),
                           batch, plan.img_h, plan.img_w, reinterpret_cast<int8_t*>(arena + plan.input.offset),
                           stream);
  }

  int enqueue(int batch, int slot = 0, bool ingress = true) {
    if (ingress)
      if (int r = enqueue_ingress(batch, slot)) return r;
    for (const auto& g : groups) {
      if (g.second - g.first == 1) {
        if (int r = enqueue_op(batch, g.first, slot)) return r;
        continue;
      }
      // fork: members after the first run on side streams, then the compute stream joins them all
      const int n = g.second - g.first;
      IXB_CUDA(cudaEventRecord(ev_fork, stream));
      for (int k = 1; k < n; ++k) IXB_CUDA(cudaStreamWaitEvent(side[k - 1], ev_fork, 0));
      if (int r = enqueue_op(batch, g.first, slot)) return r;
      for (int k = 1; k < n; ++k) {
        if (int r = enqueue_op(batch, g.first + k, slot, side[k - 1])) return r;
        IXB_CUDA(cudaEventRecord(ev_join[k - 1], side[k - 1]));
      }
      for (int k = 1; k < n; ++k) IXB_CUDA(cudaStreamWaitEvent(stream, ev_join[k - 1], 0));
    }
    return 0;
  }

  int graph_for(int batch, cudaGraphExec_t* out, int slot = 0, bool ingress = true) {
    const int key = (batch * kSlots + slot) * 2 + (ingress ? 0 : 1);
    auto it = graphs.find(key);
    if (it != graphs.end()) {
      *out = it->second;
      return 0;
    }
    cudaGraph_t g = nullptr;
    IXB_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    int r = enqueue(batch, slot, ingress);
    cudaError_t e = cudaStreamEndCapture(stream, &g);
    if (r) {
      if (g) cudaGraphDestroy(g);
      return r;
    }
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
    graphs[key] = exec;
    *out = exec;
    return 0;
  }

  bool any_busy() const {
    for (const Slot& sl : slots)
      if (sl.busy) return true;
    return false;
  }
};

// Poll an event until it completes or the timeout runs out (spin first: a step takes milliseconds).
int wait_event(cudaEvent_t ev, int timeout_ms) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return 0;
    if (e != cudaErrorNotReady) return cuda_fail(e, "run");
    const auto us = std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0);
    if (us.count() >= 1000LL * timeout_ms) return fail(IXB_ERR_TIMEOUT, "run did not finish within the timeout");
    if (us.count() < 5000) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

extern "C" {

const char* ixb_last_error(void) { return g_last_error.c_str(); }

int ixb_abi_sizes(uint64_t* sizes, int n) {
  const uint64_t v[4] = {sizeof(ixb_segment), sizeof(ixb_conv_desc), sizeof(ixb_pool_desc), sizeof(ixb_plan)};
  for (int i = 0; i < n && i < 4; ++i) sizes[i] = v[i];
  return 0;
}
int ixb_version(void) { return IXB_API_VERSION; }

int ixb_check_wait_timeout(int limit_us, void* stream) {
  if (limit_us < 1 || limit_us > 2000000) return fail(IXB_ERR_INVALID, "limit_us outside [1, 2000000]");
  if (int r = read_device_error()) return r;  // start from a clear flag
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bounded_wait_probe_kernel<<<1, 32, 0, st>>>(1000ull * (unsigned long long)limit_us);
  IXB_CUDA(cudaGetLastError());
  IXB_CUDA(cudaStreamSynchronize(st));
  return read_device_error();
}

int ixb_device_error(int* flag) {
  unsigned int v = 0;
  IXB_CUDA(cudaMemcpyFromSymbol(&v, g_dev_error, sizeof v));
  unsigned int z = 0;
  IXB_CUDA(cudaMemcpyToSymbol(g_dev_error, &z, sizeof z));
  if (flag) *flag = (int)v;
  return 0;
}

int ixb_session_create(const ixb_plan* plan, int device, void* arena, uint64_t arena_bytes, ixb_session** out) {
  if (!plan || !out) return fail(IXB_ERR_INVALID, "null plan or output pointer");
  *out = nullptr;
  if (plan->api_version != IXB_API_VERSION) return fail(IXB_ERR_INVALID, "plan api_version mismatch");
  if (plan->max_batch < 1 || plan->n_ops < 1 || plan->n_convs < 1) return fail(IXB_ERR_INVALID, "empty plan");
  if (plan->arena_bytes > arena_bytes && arena) return fail(IXB_ERR_INVALID, "arena smaller than the plan");
  auto* s = new ixb_session();  // the op list and branch groups are checked before any CUDA call
  s->device = device;
  s->plan = *plan;
  s->convs.assign(plan->convs, plan->convs + plan->n_convs);
  s->pools.assign(plan->pools, plan->pools + plan->n_pools);
  s->ops.assign(plan->ops, plan->ops + plan->n_ops);
  s->plan.convs = nullptr;
  s->plan.pools = nullptr;
  s->plan.ops = nullptr;
  for (size_t i = 0; i < s->ops.size(); ++i) {
    const ixb_op& op = s->ops[i];
    const int kind = op.kind & 0xFF;
    const bool with_prev = (op.kind & IXB_OP_WITH_PREV) != 0;
    if ((kind == IXB_OP_CONV && (op.index < 0 || op.index >= plan->n_convs)) ||
        (kind == IXB_OP_POOL && (op.index < 0 || op.index >= plan->n_pools)) ||
        (kind != IXB_OP_CONV && kind != IXB_OP_POOL) || (op.kind & ~(0xFF | IXB_OP_WITH_PREV))) {
      delete s;
      return fail(IXB_ERR_INVALID, "op list names a missing layer");
    }
    if (!with_prev) {
      s->groups.push_back({(int)i, (int)i + 1});
      continue;
    }
    if (i == 0 || kind != IXB_OP_CONV || (s->ops[i - 1].kind & 0xFF) != IXB_OP_CONV ||
        s->groups.back().second - s->groups.back().first >= IXB_MAX_BRANCHES) {
      delete s;
      return fail(IXB_ERR_INVALID, "IXB_OP_WITH_PREV joins convs only, at most IXB_MAX_BRANCHES per group");
    }
    s->groups.back().second = (int)i + 1;
  }
  // no member of a branch group may read or write what another member writes
  for (const auto& g : s->groups) {
    if (g.second - g.first < 2) continue;
    const int n = g.second - g.first;
    std::vector<std::vector<Span>> rd(n), wr(n);
    for (int k = 0; k < n; ++k) conv_spans(s->convs[s->ops[g.first + k].index], plan->max_batch, rd[k], wr[k]);
    for (int x = 0; x < n; ++x)
      for (int y = 0; y < n; ++y) {
        if (x == y) continue;
        bool hit = false;
        for (const Span& w : wr[x]) {
          for (const Span& r : rd[y]) hit = hit || spans_overlap(w, r);
          for (const Span& w2 : wr[y]) hit = hit || spans_overlap(w, w2);
        }
        if (hit) {
          const int op = g.first + std::max(x, y);
          delete s;
          return fail(IXB_ERR_INVALID, "branch group at op " + std::to_string(op) +
                                           ": a member reads or writes what another member writes");
        }
      }
  }
  if (cudaError_t e = cudaSetDevice(device)) {
    delete s;
    return cuda_fail(e, "cudaSetDevice");
  }
  s->arena_bytes = arena ? arena_bytes : plan->arena_bytes;
  if (arena) {
    s->arena = static_cast<uint8_t*>(arena);
  } else {
    cudaError_t e = cudaMalloc(&s->arena, s->arena_bytes);
    if (e == cudaSuccess) e = cudaMemset(s->arena, 0, s->arena_bytes);
    if (e != cudaSuccess) {
      delete s;
      return cuda_fail(e, "arena allocation");
    }
    s->own_arena = true;
  }
  // image staging, input lookup table, stem input and egress must lie in the arena
  std::string err;
  const int B = plan->max_batch;
  const unsigned long long img_bytes = (unsigned long long)B * 3 * plan->img_h * plan->img_w;
  int bad = 0;
  if (plan->img_w % 4 || plan->img_h < 1) bad = fail(IXB_ERR_INVALID, "image width must be a multiple of 4");
  else if (plan->images_offset % 16 || plan->images_offset + img_bytes > s->arena_bytes)
    bad = fail(IXB_ERR_INVALID, "image staging outside the arena");
  else if (plan->input_lut_offset + 256 > s->arena_bytes) bad = fail(IXB_ERR_INVALID, "input table outside the arena");
  else if (check_seg(plan->input, B, s->arena_bytes, true, "stem input", err)) bad = fail(IXB_ERR_INVALID, err);
  else if (plan->input.height != plan->img_h || plan->input.width != plan->img_w || plan->input.channels != 3)
    bad = fail(IXB_ERR_INVALID, "stem input view must be the img_h x img_w 3-channel image");
  else if (plan->input_s2d &&
           (plan->img_h % 2 || check_seg(plan->input_s2d_view, B, s->arena_bytes, false, "stem space-to-depth input", err)))
    bad = fail(IXB_ERR_INVALID, plan->img_h % 2 ? "a space-to-depth stem input needs an even image height" : err.c_str());
  else if (plan->input_s2d &&
           (plan->input_s2d_view.height != plan->img_h / 2 || plan->input_s2d_view.width != plan->img_w / 2 ||
            plan->input_s2d_view.channels != 16 || plan->input_s2d_view.up2 || plan->input_s2d_view.chunk_offset))
    bad = fail(IXB_ERR_INVALID, "the stem's space-to-depth view must be one chunk of (img_h/2) x (img_w/2)");
  else if (plan->egress_offset + (unsigned long long)B * plan->egress_image_bytes > s->arena_bytes)
    bad = fail(IXB_ERR_INVALID, "egress outside the arena");
  else if (plan->extra_slots < 0 || plan->extra_slots > IXB_MAX_EXTRA_SLOTS)
    bad = fail(IXB_ERR_INVALID, "extra_slots outside [0, IXB_MAX_EXTRA_SLOTS]");
  for (int i = 0; !bad && i < plan->extra_slots; ++i)
    if (plan->extra_images_offset[i] % 16 || plan->extra_images_offset[i] + img_bytes > s->arena_bytes ||
        plan->extra_egress_offset[i] + (unsigned long long)B * plan->egress_image_bytes > s->arena_bytes)
      bad = fail(IXB_ERR_INVALID, "pipeline slot " + std::to_string(i + 1) + " outside the arena");
  if (!bad) bad = s->prepare(B);
  if (bad) {
    if (s->own_arena) cudaFree(s->arena);
    delete s;
    return bad;
  }
  cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->d2h, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreate(&s->ev0);
  if (e == cudaSuccess) e = cudaEventCreate(&s->ev1);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->ev_done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->ev_fork, cudaEventDisableTiming);
  for (int k = 0; k < IXB_MAX_BRANCHES - 1; ++k) {
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->side[k], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s->ev_join[k], cudaEventDisableTiming);
  }
  for (auto& sl : s->slots) {
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sl.h2d_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreate(&sl.t0);
    if (e == cudaSuccess) e = cudaEventCreate(&sl.t1);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sl.d2h_done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreate(&sl.pre0);
    if (e == cudaSuccess) e = cudaEventCreate(&sl.post1);
  }
  if (e != cudaSuccess) {
    int r = cuda_fail(e, "stream/event creation");
    ixb_session_destroy(s);
    return r;
  }
  // branch-group shares from measured member times, then the launches rebuild with them
  int r = s->measure_costs(B);
  if (!r) r = s->prepare(B);
  if (r) {
    ixb_session_destroy(s);
    return r;
  }
  *out = s;
  return 0;
}

int ixb_session_destroy(ixb_session* s) {
  if (!s) return 0;
  cudaSetDevice(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  if (s->h2d) cudaStreamSynchronize(s->h2d);
  if (s->d2h) cudaStreamSynchronize(s->d2h);
  for (auto& kv : s->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& sl : s->slots) {
    for (cudaEvent_t ev : {sl.h2d_done, sl.t0, sl.t1, sl.d2h_done, sl.pre0, sl.post1})
      if (ev) cudaEventDestroy(ev);
    if (sl.frames_dev) cudaFree(sl.frames_dev);
  }
  if (s->det_tables) cudaFree(s->det_tables);
  if (s->det_mem) cudaFree(s->det_mem);
  if (s->det_pinned) cudaFreeHost(s->det_pinned);
  if (s->h2d) cudaStreamDestroy(s->h2d);
  if (s->d2h) cudaStreamDestroy(s->d2h);
  if (s->ev0) cudaEventDestroy(s->ev0);
  if (s->ev1) cudaEventDestroy(s->ev1);
  if (s->ev_done) cudaEventDestroy(s->ev_done);
  for (int k = 0; k < IXB_MAX_BRANCHES - 1; ++k) {
    if (s->side[k]) cudaStreamSynchronize(s->side[k]);
    if (s->side[k]) cudaStreamDestroy(s->side[k]);
    if (s->ev_join[k]) cudaEventDestroy(s->ev_join[k]);
  }
  if (s->ev_fork) cudaEventDestroy(s->ev_fork);
  if (s->stream) cudaStreamDestroy(s->stream);
  if (s->own_arena && s->arena) cudaFree(s->arena);
  delete s;
  return 0;
}

void* ixb_session_arena(ixb_session* s) { return s ? s->arena : nullptr; }
void* ixb_session_stream(ixb_session* s) { return s ? (void*)s->stream : nullptr; }

int ixb_session_launches(ixb_session* s, int batch) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  (void)batch;
  return 1 + (int)s->ops.size();
}

int ixb_session_run(ixb_session* s, const uint8_t* images, int batch, int8_t* egress, int flags) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  if (batch < 1 || batch > s->plan.max_batch) return fail(IXB_ERR_INVALID, "batch outside [1, max_batch]");
  // a run while an asynchronous one is pending queues behind it on the same stream; the wait covers both
  if (s->any_busy()) return fail(IXB_ERR_INVALID, "submitted runs are still in flight");
  const bool in_store = (flags & IXB_IN_STORE) != 0;
  if (!(flags & IXB_IN_DEVICE) && !in_store && !images) return fail(IXB_ERR_INVALID, "null images");
  if (in_store && images) return fail(IXB_ERR_INVALID, "IXB_IN_STORE runs take no images");
  if (!(flags & IXB_OUT_DEVICE) && !egress) return fail(IXB_ERR_INVALID, "null egress");
  const bool copy_in = images != nullptr, copy_out = egress != nullptr;
  IXB_CUDA(cudaSetDevice(s->device));
  if (int r = s->prepare(batch)) return r;
  const size_t in_bytes = (size_t)batch * 3 * s->plan.img_h * s->plan.img_w;
  if (copy_in)
    IXB_CUDA(cudaMemcpyAsync(s->arena + s->plan.images_offset, images, in_bytes,
                             (flags & IXB_IN_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                             s->stream));
  IXB_CUDA(cudaEventRecord(s->ev0, s->stream));
  if (flags & IXB_NO_GRAPH) {
    if (int r = s->enqueue(batch, 0, !in_store)) return r;
  } else {
    cudaGraphExec_t exec;
    if (int r = s->graph_for(batch, &exec, 0, !in_store)) return r;
    IXB_CUDA(cudaGraphLaunch(exec, s->stream));
  }
  IXB_CUDA(cudaEventRecord(s->ev1, s->stream));
  if (copy_out)
    IXB_CUDA(cudaMemcpyAsync(egress, s->arena + s->plan.egress_offset, (size_t)batch * s->plan.egress_image_bytes,
                             (flags & IXB_OUT_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost,
                             s->stream));
  IXB_CUDA(cudaEventRecord(s->ev_done, s->stream));
  s->pending = true;
  if (flags & IXB_ASYNC) return 0;
  return ixb_session_wait(s, 60000);
}

int ixb_session_wait(ixb_session* s, int timeout_ms) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  if (!s->pending) return 0;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(s->ev_done);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) {
      s->pending = false;
      return cuda_fail(e, "run");
    }
    const auto us = std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0);
    if (us.count() >= 1000LL * timeout_ms) return fail(IXB_ERR_TIMEOUT, "run did not finish within the timeout");
    // spin briefly (a step takes milliseconds), then back off
    if (us.count() < 5000) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  s->pending = false;
  cudaEventElapsedTime(&s->last_ms, s->ev0, s->ev1);
  return read_device_error();
}

int ixb_session_submit(ixb_session* s, const uint8_t* images, int batch, int8_t* egress, uint64_t* ticket) {
  if (!s || !images || !egress || !ticket) return fail(IXB_ERR_INVALID, "null argument");
  if (batch < 1 || batch > s->plan.max_batch) return fail(IXB_ERR_INVALID, "batch outside [1, max_batch]");
  if (s->pending) return fail(IXB_ERR_INVALID, "a synchronous run is pending");
  IXB_CUDA(cudaSetDevice(s->device));
  const uint64_t t = s->next_ticket;
  const int slot = s->slot_of(t);
  ixb_session::Slot& sl = s->slots[slot];
  if (sl.busy)  // the run `depth` tickets back still owns this slot's buffers
    if (int r = ixb_session_wait_ticket(s, sl.ticket, 60000)) return r;
  if (int r = s->prepare(batch, slot)) return r;
  cudaGraphExec_t exec;
  if (int r = s->graph_for(batch, &exec, slot)) return r;
  const size_t in_bytes = (size_t)batch * 3 * s->plan.img_h * s->plan.img_w;
  IXB_CUDA(cudaMemcpyAsync(s->arena + s->images_at(slot), images, in_bytes, cudaMemcpyDefault, s->h2d));
  IXB_CUDA(cudaEventRecord(sl.h2d_done, s->h2d));
  IXB_CUDA(cudaStreamWaitEvent(s->stream, sl.h2d_done, 0));
  IXB_CUDA(cudaEventRecord(sl.t0, s->stream));
  IXB_CUDA(cudaGraphLaunch(exec, s->stream));
  IXB_CUDA(cudaEventRecord(sl.t1, s->stream));
  IXB_CUDA(cudaStreamWaitEvent(s->d2h, sl.t1, 0));
  IXB_CUDA(cudaMemcpyAsync(egress, s->arena + s->egress_at(slot), (size_t)batch * s->plan.egress_image_bytes,
                           cudaMemcpyDefault, s->d2h));
  IXB_CUDA(cudaEventRecord(sl.d2h_done, s->d2h));
  sl.ticket = t;
  sl.busy = true;
  sl.detections = false;
  s->next_ticket = t + 1;
  *ticket = t;
  return 0;
}

int ixb_session_wait_ticket(ixb_session* s, uint64_t ticket, int timeout_ms) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  if (ticket == 0 || ticket >= s->next_ticket) return fail(IXB_ERR_INVALID, "unknown ticket");
  ixb_session::Slot& sl = s->slots[s->slot_of(ticket)];
  if (!sl.busy || sl.ticket != ticket) return 0;  // already completed and collected
  if (int r = wait_event(sl.d2h_done, timeout_ms)) return r;
  sl.busy = false;
  cudaEventElapsedTime(&s->last_ms, sl.t0, sl.t1);
  if (sl.detections) {  // the stages of a detection run, as the reference's ignite_timings_t
    float pre = 0.f, post = 0.f;
    cudaEventElapsedTime(&pre, sl.pre0, sl.t0);
    cudaEventElapsedTime(&post, sl.t1, sl.post1);
    s->last_timings.preprocess_ms = sl.frames ? pre : 0.0;
    s->last_timings.gpu_exec_ms = s->last_ms;
    s->last_timings.postprocess_ms = post;
    s->last_timings.glass_to_glass_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - sl.submitted).count();
  }
  return read_device_error();
}

// ---------------------------------------------------------------- detection stage
int ixb_session_set_detect(ixb_session* s, const ixb_detect_config* cfg) {
  if (!s || !cfg) return fail(IXB_ERR_INVALID, "null argument");
  if (s->pending || s->any_busy()) return fail(IXB_ERR_INVALID, "runs are still in flight");
  if (cfg->capacity < 1 || cfg->capacity > kDecodeMaxAnchors) return fail(IXB_ERR_INVALID, "capacity outside [1, 8400]");
  for (int h = 0; h < 3; ++h)
    if (!(cfg->cls_scale[h] > 0.f)) return fail(IXB_ERR_INVALID, "class head scales must be positive");
  IXB_CUDA(cudaSetDevice(s->device));
  DecodeParams p;
  if (int r = prepare_decode(cfg->decode, s->plan.egress_image_bytes, p)) return r;
  // the tables' ranks and DFL checks once, here, instead of in every decode launch (the session
  // reads the caller's tables from here on; a change to them goes through set_detect again)
  if (!s->det_tables) IXB_CUDA(cudaMalloc(&s->det_tables, 2 * kScoreVals + 16));
  p.ranks = reinterpret_cast<const uint16_t*>(s->det_tables);
  p.toe = reinterpret_cast<const int32_t*>(s->det_tables + 2 * kScoreVals);
  decode_tables_kernel<<<1, kDecodeThreads, 0, s->stream>>>(p, reinterpret_cast<uint16_t*>(s->det_tables),
                                                            reinterpret_cast<int32_t*>(s->det_tables + 2 * kScoreVals));
  IXB_CUDA(cudaGetLastError());
  IXB_CUDA(cudaStreamSynchronize(s->stream));
  const bool grow = !s->detect || cfg->capacity != s->dcfg.capacity;
  s->dcfg = *cfg;
  s->dparams = p;
  if (grow) {
    if (s->det_mem) cudaFree(s->det_mem);
    if (s->det_pinned) cudaFreeHost(s->det_pinned);
    s->det_mem = s->det_pinned = nullptr;
    s->detect = false;
    const size_t per = s->det_slot_bytes();
    IXB_CUDA(cudaMalloc(&s->det_mem, per * ixb_session::kSlots));
    IXB_CUDA(cudaMallocHost(&s->det_pinned, per * ixb_session::kSlots));
    for (int k = 0; k < ixb_session::kSlots; ++k) {
      ixb_session::Slot& sl = s->slots[k];
      sl.det_dev = s->det_mem + k * per;
      sl.det_host = s->det_pinned + k * per;
      sl.lb_dev = reinterpret_cast<float*>(sl.det_dev + per - s->lb_bytes());
      sl.lb_host = reinterpret_cast<float*>(sl.det_host + per - s->lb_bytes());
      sl.detections = false;
    }
  }
  s->detect = true;
  return 0;
}

int ixb_session_set_thresholds(ixb_session* s, float conf, float iou) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  if (!s->detect) return fail(IXB_ERR_INVALID, "the session has no detection stage (ixb_session_set_detect)");
  if (!(conf > 0.f && conf < 1.f) || !(iou >= 0.f && iou <= 1.f))
    return fail(IXB_ERR_INVALID, "conf must lie in (0, 1) and iou in [0, 1]");
  if (s->pending || s->any_busy()) return fail(IXB_ERR_INVALID, "runs are still in flight");
  ixb_detect_config c = s->dcfg;
  // the prune threshold on a class head's int8 logit: logit(conf) / scale + zero point
  const double cc = std::min(std::max((double)conf, 1e-12), 1.0 - 1e-12);
  for (int h = 0; h < 3; ++h)
    c.decode.head[h].q_threshold = std::log(cc / (1.0 - cc)) / (double)c.cls_scale[h] + (double)c.cls_zero_point[h];
  c.decode.conf = conf;
  c.decode.iou = iou;
  return ixb_session_set_detect(s, &c);
}

int ixb_session_set_class_names(ixb_session* s, const char* const* names, int n) {
  if (!s || n < 0 || (n > 0 && !names)) return fail(IXB_ERR_INVALID, "bad class names");
  s->class_names.clear();
  for (int i = 0; i < n; ++i) s->class_names.emplace_back(names[i] ? names[i] : "");
  return 0;
}

}  // extern "C"

namespace {
// Claims the ticket's slot for a detection run: waits for the run `depth` tickets back, builds the
// launches and the graph. Returns the slot.
int claim_detect_slot(ixb_session* s, int batch, bool ingress, cudaGraphExec_t* exec, int* slot_out) {
  if (!s->detect) return fail(IXB_ERR_INVALID, "the session has no detection stage (ixb_session_set_detect)");
  if (batch < 1 || batch > s->plan.max_batch) return fail(IXB_ERR_INVALID, "batch outside [1, max_batch]");
  if (s->pending) return fail(IXB_ERR_INVALID, "a synchronous run is pending");
  IXB_CUDA(cudaSetDevice(s->device));
  const int slot = s->slot_of(s->next_ticket);
  ixb_session::Slot& sl = s->slots[slot];
  if (sl.busy)
    if (int r = ixb_session_wait_ticket(s, sl.ticket, 60000)) return r;
  if (int r = s->prepare(batch, slot)) return r;
  if (int r = s->graph_for(batch, exec, slot, ingress)) return r;
  *slot_out = slot;
  return 0;
}

// After the graph on the compute stream: decode + NMS into the slot's detections, then one copy back.
int enqueue_detect_tail(ixb_session* s, int slot, int batch, uint64_t* ticket) {
  ixb_session::Slot& sl = s->slots[slot];
  DecodeParams p = s->dparams;
  p.egress = reinterpret_cast<const int8_t*>(s->arena + s->egress_at(slot));
  p.letterbox = sl.lb_dev;
  p.capacity = s->dcfg.capacity;
  s->det_layout(sl.det_dev, batch, &p.out_count, &p.out_box, &p.out_score, &p.out_class);
  if (int r = launch_decode(p, batch, s->stream)) return r;
  IXB_CUDA(cudaEventRecord(sl.post1, s->stream));
  IXB_CUDA(cudaStreamWaitEvent(s->d2h, sl.post1, 0));
  IXB_CUDA(cudaMemcpyAsync(sl.det_host, sl.det_dev, s->det_bytes(batch), cudaMemcpyDeviceToHost, s->d2h));
  IXB_CUDA(cudaEventRecord(sl.d2h_done, s->d2h));
  const uint64_t t = s->next_ticket;
  sl.ticket = t;
  sl.busy = true;
  sl.detections = true;
  sl.batch = batch;
  s->next_ticket = t + 1;
  *ticket = t;
  return 0;
}
}  // namespace

extern "C" {

int ixb_session_submit_detect(ixb_session* s, const uint8_t* images, int batch, const float* letterbox,
                              uint64_t* ticket) {
  if (!s || !images || !ticket) return fail(IXB_ERR_INVALID, "null argument");
  cudaGraphExec_t exec;
  int slot = 0;
  if (int r = claim_detect_slot(s, batch, true, &exec, &slot)) return r;
  ixb_session::Slot& sl = s->slots[slot];
  sl.submitted = std::chrono::steady_clock::now();
  sl.frames = false;
  for (int i = 0; i < batch; ++i) {
    sl.lb_host[3 * i] = letterbox ? letterbox[3 * i] : 0.f;
    sl.lb_host[3 * i + 1] = letterbox ? letterbox[3 * i + 1] : 0.f;
    sl.lb_host[3 * i + 2] = letterbox ? letterbox[3 * i + 2] : 1.f;
  }
  const size_t in_bytes = (size_t)batch * 3 * s->plan.img_h * s->plan.img_w;
  IXB_CUDA(cudaMemcpyAsync(s->arena + s->images_at(slot), images, in_bytes, cudaMemcpyDefault, s->h2d));
  IXB_CUDA(cudaMemcpyAsync(sl.lb_dev, sl.lb_host, (size_t)batch * 12, cudaMemcpyHostToDevice, s->h2d));
  IXB_CUDA(cudaEventRecord(sl.h2d_done, s->h2d));
  IXB_CUDA(cudaStreamWaitEvent(s->stream, sl.h2d_done, 0));
  IXB_CUDA(cudaEventRecord(sl.pre0, s->stream));
  IXB_CUDA(cudaEventRecord(sl.t0, s->stream));
  IXB_CUDA(cudaGraphLaunch(exec, s->stream));
  IXB_CUDA(cudaEventRecord(sl.t1, s->stream));
  return enqueue_detect_tail(s, slot, batch, ticket);
}

int ixb_session_submit_frames(ixb_session* s, const uint8_t* frames, int batch, int src_w, int src_h, int src_stride,
                              uint64_t frame_bytes, uint64_t* ticket) {
  if (!s || !frames || !ticket) return fail(IXB_ERR_INVALID, "null argument");
  if (src_w < 1 || src_h < 1 || src_stride < 3 * src_w ||
      (batch > 1 && frame_bytes < (uint64_t)src_stride * (src_h - 1) + 3ull * src_w))
    return fail(IXB_ERR_INVALID, "frame sizes and strides do not hold the frames");
  cudaGraphExec_t exec;
  int slot = 0;
  if (int r = claim_detect_slot(s, batch, false, &exec, &slot)) return r;
  ixb_session::Slot& sl = s->slots[slot];
  sl.submitted = std::chrono::steady_clock::now();
  sl.frames = true;
  const size_t need = (size_t)(batch - 1) * frame_bytes + (size_t)src_stride * (src_h - 1) + 3ull * src_w;
  if (need > sl.frames_cap) {  // the slot's previous run has completed (claim_detect_slot)
    if (sl.frames_dev) cudaFree(sl.frames_dev);
    sl.frames_dev = nullptr;
    sl.frames_cap = 0;
    IXB_CUDA(cudaMalloc(&sl.frames_dev, need));
    sl.frames_cap = need;
  }
  IXB_CUDA(cudaMemcpyAsync(sl.frames_dev, frames, need, cudaMemcpyDefault, s->h2d));
  IXB_CUDA(cudaEventRecord(sl.h2d_done, s->h2d));
  IXB_CUDA(cudaStreamWaitEvent(s->stream, sl.h2d_done, 0));
  IXB_CUDA(cudaEventRecord(sl.pre0, s->stream));
  const ixb_plan& pl = s->plan;
  const int row = pl.img_w + 4;
  int8_t* base = reinterpret_cast<int8_t*>(s->arena + pl.input.offset) + ((long long)row + 1) * 8;
  float lb[3];
  if (int r = ixb_letterbox_frames(sl.frames_dev, batch, src_w, src_h, src_stride, batch > 1 ? frame_bytes : need,
                                   reinterpret_cast<const int8_t*>(s->arena + pl.input_lut_offset), base, pl.img_w,
                                   pl.img_h, row, (uint64_t)(pl.img_h + 2) * row * 8, lb, s->stream))
    return r;
  if (pl.input_s2d)
    if (int r = launch_ingress_s2d(nullptr, reinterpret_cast<const int8_t*>(s->arena + pl.input.offset), nullptr, batch,
                                   pl.img_h, pl.img_w, s->arena, pl.input_s2d_view, s->stream))
      return r;
  for (int i = 0; i < batch; ++i)
    for (int j = 0; j < 3; ++j) sl.lb_host[3 * i + j] = lb[j];
  IXB_CUDA(cudaMemcpyAsync(sl.lb_dev, sl.lb_host, (size_t)batch * 12, cudaMemcpyHostToDevice, s->stream));
  IXB_CUDA(cudaEventRecord(sl.t0, s->stream));
  IXB_CUDA(cudaGraphLaunch(exec, s->stream));
  IXB_CUDA(cudaEventRecord(sl.t1, s->stream));
  return enqueue_detect_tail(s, slot, batch, ticket);
}

int ixb_session_detections(ixb_session* s, uint64_t ticket, int timeout_ms, int32_t* batch, const int32_t** counts,
                           const float** boxes, const float** scores, const int32_t** classes) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  if (int r = ixb_session_wait_ticket(s, ticket, timeout_ms)) return r;
  const ixb_session::Slot& sl = s->slots[s->slot_of(ticket)];
  if (sl.ticket != ticket) return fail(IXB_ERR_INVALID, "a later run has reused this ticket's slot");
  if (!sl.detections) return fail(IXB_ERR_INVALID, "the ticket's run returned heads, not detections");
  int32_t* c;
  float *b, *sc;
  int32_t* cl;
  s->det_layout(sl.det_host, sl.batch, &c, &b, &sc, &cl);
  if (batch) *batch = sl.batch;
  if (counts) *counts = c;
  if (boxes) *boxes = b;
  if (scores) *scores = sc;
  if (classes) *classes = cl;
  return 0;
}

int ixb_session_wait_detections(ixb_session* s, uint64_t ticket, int timeout_ms, int image, ixb_detection* out,
                                int max_detections) {
  int32_t batch = 0;
  const int32_t* counts;
  const float *boxes, *scores;
  const int32_t* classes;
  if (int r = ixb_session_detections(s, ticket, timeout_ms, &batch, &counts, &boxes, &scores, &classes)) return r;
  if (image < 0 || image >= batch) return fail(IXB_ERR_INVALID, "image outside the run's batch");
  const int n = counts[image];
  if (n < 0)
    return fail(IXB_ERR_CAPACITY, "more detections survive NMS than the session's capacity (" +
                                      std::to_string(s->dcfg.capacity) + ")");
  if (max_detections > 0 && !out) return fail(IXB_ERR_INVALID, "null detections array");
  const int m = std::min(n, std::max(max_detections, 0));
  const size_t cap = (size_t)s->dcfg.capacity;
  for (int k = 0; k < m; ++k) {
    const size_t o = (size_t)image * cap + k;
    ixb_detection& d = out[k];
    d.x0 = boxes[4 * o];
    d.y0 = boxes[4 * o + 1];
    d.w = boxes[4 * o + 2];
    d.h = boxes[4 * o + 3];
    d.score = scores[o];
    d.class_id = classes[o];
    memset(d.class_name, 0, sizeof d.class_name);
    if (d.class_id >= 0 && d.class_id < (int)s->class_names.size())
      strncpy(d.class_name, s->class_names[d.class_id].c_str(), sizeof d.class_name - 1);
  }
  return m;
}

int ixb_run_frame(ixb_session* s, const uint8_t* bgr, int width, int height, int stride, ixb_detection* out,
                  int max_detections) {
  uint64_t t = 0;
  if (int r = ixb_session_submit_frames(s, bgr, 1, width, height, stride, (uint64_t)stride * height, &t)) return r;
  return ixb_session_wait_detections(s, t, 60000, 0, out, max_detections);
}

int ixb_session_last_timings(ixb_session* s, ixb_timings* t) {
  if (!s || !t) return fail(IXB_ERR_INVALID, "null argument");
  *t = s->last_timings;
  return 0;
}

int ixb_session_streams(ixb_session* s, void** compute, void** h2d, void** d2h) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  if (compute) *compute = s->stream;
  if (h2d) *h2d = s->h2d;
  if (d2h) *d2h = s->d2h;
  return 0;
}

int ixb_session_last_ms(ixb_session* s, float* ms) {
  if (!s || !ms) return fail(IXB_ERR_INVALID, "null argument");
  *ms = s->last_ms;
  return 0;
}

int ixb_session_trace(ixb_session* s, int batch, int iters, uint64_t* ns) {
  if (!s || !ns || iters < 1) return fail(IXB_ERR_INVALID, "bad trace arguments");
  if (batch < 1 || batch > s->plan.max_batch) return fail(IXB_ERR_INVALID, "batch outside [1, max_batch]");
  if (s->pending) return fail(IXB_ERR_INVALID, "a run is pending");
  if (s->any_busy()) return fail(IXB_ERR_INVALID, "submitted runs are still in flight");
  IXB_CUDA(cudaSetDevice(s->device));
  if (int r = s->prepare(batch)) return r;
  const size_t n = s->ops.size();
  const int key = batch * ixb_session::kSlots;
  unsigned long long* buf = nullptr;
  IXB_CUDA(cudaMalloc(&buf, n * 3 * sizeof(unsigned long long)));
  std::vector<unsigned long long> init(n * 3);
  for (size_t i = 0; i < n; ++i) {
    init[3 * i] = init[3 * i + 1] = ~0ull;
    init[3 * i + 2] = 0;
  }
  // a traced copy of the launches, captured into its own graph (the session's graphs stay as they are)
  std::vector<ConvLaunch> traced = s->conv_launch[key];
  for (size_t i = 0; i < n; ++i)
    if ((s->ops[i].kind & 0xFF) == IXB_OP_CONV) traced[s->ops[i].index].p.trace = buf + 3 * i;
  std::swap(s->conv_launch[key], traced);
  cudaGraph_t g = nullptr;
  cudaGraphExec_t exec = nullptr;
  int rc = 0;
  cudaError_t e = cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    rc = s->enqueue(batch, 0, true);
    e = cudaStreamEndCapture(s->stream, &g);
  }
  std::swap(s->conv_launch[key], traced);
  if (!rc && e == cudaSuccess) e = cudaGraphInstantiate(&exec, g, 0);
  if (g) cudaGraphDestroy(g);
  for (int it = 0; it < iters && !rc && e == cudaSuccess; ++it) {
    e = cudaMemcpyAsync(buf, init.data(), init.size() * sizeof(unsigned long long), cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
  }
  if (!rc && e == cudaSuccess)
    e = cudaMemcpy(init.data(), buf, init.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
  if (exec) cudaGraphExecDestroy(exec);
  cudaFree(buf);
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "trace run");
  for (size_t i = 0; i < n * 3; ++i) ns[i] = (init[i] == ~0ull) ? 0 : init[i];
  return read_device_error();
}

int ixb_session_profile(ixb_session* s, int batch, int iters, float* ms) {
  if (!s || !ms || iters < 1) return fail(IXB_ERR_INVALID, "bad profile arguments");
  if (batch < 1 || batch > s->plan.max_batch) return fail(IXB_ERR_INVALID, "batch outside [1, max_batch]");
  if (s->pending) return fail(IXB_ERR_INVALID, "a run is pending");
  if (s->any_busy()) return fail(IXB_ERR_INVALID, "submitted runs are still in flight");
  IXB_CUDA(cudaSetDevice(s->device));
  if (int r = s->prepare(batch)) return r;
  const size_t n = s->ops.size();
  std::vector<cudaEvent_t> ev(n + 1);
  for (auto& e : ev) IXB_CUDA(cudaEventCreate(&e));
  std::vector<double> acc(n, 0.0);
  int rc = 0;
  for (int it = 0; it < iters && !rc; ++it) {
    rc = s->enqueue_ingress(batch);
    if (!rc) rc = cudaEventRecord(ev[0], s->stream) == cudaSuccess ? 0 : fail(IXB_ERR_CUDA, "event record");
    for (size_t i = 0; i < n && !rc; ++i) {
      rc = s->enqueue_op(batch, (int)i);
      if (!rc && cudaEventRecord(ev[i + 1], s->stream) != cudaSuccess) rc = fail(IXB_ERR_CUDA, "event record");
    }
    if (!rc && cudaEventSynchronize(ev[n]) != cudaSuccess) rc = fail(IXB_ERR_CUDA, "event synchronize");
    for (size_t i = 0; i < n && !rc; ++i) {
      float t = 0.f;
      cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
      acc[i] += t;
    }
  }
  for (auto& e : ev) cudaEventDestroy(e);
  if (rc) return rc;
  for (size_t i = 0; i < n; ++i) ms[i] = (float)(acc[i] / iters);
  return read_device_error();
}

int ixb_conv_layer(const ixb_conv_desc* d, void* arena, uint64_t arena_bytes, int batch, void* stream) {
  if (!d || !arena) return fail(IXB_ERR_INVALID, "null argument");
  ConvLaunch L;
  std::string err;
  if (prepare_conv(*d, static_cast<uint8_t*>(arena), arena_bytes, batch, L, err)) return fail(IXB_ERR_INVALID, err);
  return launch_conv(L, static_cast<cudaStream_t>(stream));
}

int ixb_conv_layer_stats(const ixb_conv_desc* d, void* arena, uint64_t arena_bytes, int batch, void* stream,
                         uint64_t* stats, int64_t stats_words) {
  if (!d || !arena || !stats) return fail(IXB_ERR_INVALID, "null argument");
  ConvLaunch L;
  std::string err;
  if (prepare_conv(*d, static_cast<uint8_t*>(arena), arena_bytes, batch, L, err)) return fail(IXB_ERR_INVALID, err);
  if ((int64_t)L.grid.x * L.grid.y * kStatWords > stats_words) return fail(IXB_ERR_INVALID, "stats buffer too small");
  L.p.stats = reinterpret_cast<unsigned long long*>(stats);
  return launch_conv(L, static_cast<cudaStream_t>(stream));
}

int ixb_conv_schedule(const ixb_conv_desc* d, int32_t* kb_out, int max_kb, int32_t* ops_out, int max_ops) {
  if (!d || !kb_out || !ops_out) return fail(IXB_ERR_INVALID, "null argument");
  int chunks = 0;
  for (int i = 0; i < d->nseg && i < IXB_MAX_SEGS; ++i) chunks += (d->seg[i].channels + 15) / 16;
  if (d->mode == IXB_MODE_STEM) chunks = 1;
  if (d->n_tile < 16 || d->k < 1 || d->cp < 1 || d->mode < 0 || d->mode > IXB_MODE_IM2COL)
    return fail(IXB_ERR_INVALID, "bad conv shape");
  std::vector<SchedKB> kbs;
  std::vector<SchedOp> ops;
  build_schedule(*d, chunks, kbs, ops);
  if ((int)kbs.size() > max_kb || (int)ops.size() > max_ops) return fail(IXB_ERR_INVALID, "schedule buffers too small");
  for (size_t i = 0; i < kbs.size(); ++i) {
    const SchedKB& k = kbs[i];
    const int32_t v[8] = {k.chunk0, k.nchunks, k.tap0, k.ntaps, k.op0, k.nops, k.b_off, k.b_bytes};
    for (int j = 0; j < 8; ++j) kb_out[8 * i + j] = v[j];
  }
  for (size_t i = 0; i < ops.size(); ++i) {
    const SchedOp& o = ops[i];
    const int32_t v[6] = {o.slot0, o.chunk0, o.tap0, o.slot1, o.chunk1, o.tap1};
    for (int j = 0; j < 6; ++j) ops_out[6 * i + j] = v[j];
  }
  return (int)kbs.size();
}

int ixb_conv_launch_info(const ixb_conv_desc* d, uint64_t arena_bytes, int batch, int32_t* info, int n) {
  if (!d || !info) return fail(IXB_ERR_INVALID, "null argument");
  ConvLaunch L;
  std::string err;
  // offsets are checked against arena_bytes; a null base only feeds pointer arithmetic
  if (build_conv(*d, nullptr, arena_bytes, batch, L, err)) return fail(IXB_ERR_INVALID, err);
  const int32_t v[12] = {L.p.mt, L.p.tile_rows, L.p.m_tiles, L.p.stages, L.p.b_resident, (int32_t)L.grid.x,
                         (int32_t)L.grid.y, L.smem, L.p.tmem_cols, L.p.kblocks, L.p.rowsA, L.p.cp};
  for (int i = 0; i < n && i < 12; ++i) info[i] = v[i];
  return 0;
}

int ixb_pool_layer(const ixb_pool_desc* d, void* arena, uint64_t arena_bytes, int batch, void* stream) {
  if (!d || !arena) return fail(IXB_ERR_INVALID, "null argument");
  PoolLaunch L;
  std::string err;
  if (build_pool(*d, static_cast<uint8_t*>(arena), arena_bytes, batch, L, err)) return fail(IXB_ERR_INVALID, err);
  return launch_pool(L, static_cast<cudaStream_t>(stream));
}

int ixb_i8gemm_srs(const int8_t* a, const int8_t* b, const int32_t* bias, int8_t* out, int M, int N, int K, int shift,
                   void* stream) {
  return run_i8gemm(a, b, bias, out, nullptr, M, N, K, shift, GEMM_OUT_SRS, stream);
}

int ixb_i8gemm_i32(const int8_t* a, const int8_t* b, int32_t* out, int M, int N, int K, void* stream) {
  return run_i8gemm(a, b, nullptr, nullptr, out, M, N, K, 0, GEMM_OUT_I32, stream);
}

int ixb_w4a8_image_bytes(int K, int N, uint64_t* bytes) {
  if (!bytes) return fail(IXB_ERR_INVALID, "null argument");
  if (int r = check_w4a8_shape(N, K)) return r;
  *bytes = w4a8_image_bytes(K, N);
  return 0;
}

int ixb_w4a8_prepare(const uint8_t* w_kn, const int8_t* gpos, int K, int N, uint8_t* image, void* stream) {
  if (!w_kn || !gpos || !image) return fail(IXB_ERR_INVALID, "null argument");
  if (int r = check_w4a8_shape(N, K)) return r;
  if (!aligned16(image)) return fail(IXB_ERR_INVALID, "the weight image must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  IXB_CUDA(cudaStreamSynchronize(st));
  if (int r = read_device_error()) return r;  // start from a clear flag
  const long long words = (long long)N * (K / 8);
  const int blocks = (int)std::min<long long>((words + 255) / 256, 148LL * 32);
  w4a8_pack_kernel<<<blocks, 256, 0, st>>>(w_kn, K, N, image);
  IXB_CUDA(cudaGetLastError());
  w4a8_groups_kernel<<<(N + 255) / 256, 256, 0, st>>>(gpos, K / kW4Group, N, image + (uint64_t)N * (K / 2));
  IXB_CUDA(cudaGetLastError());
  IXB_CUDA(cudaStreamSynchronize(st));
  if (int r = read_device_error())
    return r == IXB_ERR_INVALID ? fail(r, "a column's group positions span more than 4 (max - min > 4)") : r;
  return 0;
}

int ixb_w4a8_gemm(const int8_t* a, const uint8_t* image, const int32_t* shift, int8_t* out, int M, int N, int K,
                  void* stream) {
  if (!a || !image || !shift || !out) return fail(IXB_ERR_INVALID, "null argument");
  if (int r = check_w4a8_shape(N, K)) return r;
  if (!aligned16(a) || !aligned16(image) || !aligned16(out) || !aligned16(shift))
    return fail(IXB_ERR_INVALID, "W4A8 operands must be 16-byte aligned");
  GemmLaunch L;
  std::string err;
  if (plan_gemm(L, M, N, K, err, GEMM_B_W4)) return fail(IXB_ERR_INVALID, err);
  L.p.out_kind = GEMM_OUT_SRS;
  L.p.out8 = out;
  L.p.shift_vec = shift;
  L.p.wq = image;
  L.p.eg = image + (uint64_t)N * (K / 2);
  if (encode_kmajor(&L.p.ta, a, M, K, 128, err)) return fail(IXB_ERR_CUDA, err);
  if (encode_w4(&L.p.tb, image, N, K, L.p.bn, err)) return fail(IXB_ERR_CUDA, err);
  return launch_gemm<GEMM_B_W4>(L, static_cast<cudaStream_t>(stream));
}

int ixb_u8i4_gemm_i32(const uint8_t* a, const uint8_t* image, int32_t* out, int M, int N, int K, void* stream) {
  if (!a || !image || !out) return fail(IXB_ERR_INVALID, "null argument");
  if (int r = check_w4a8_shape(N, K)) return r;
  if (K > 32768) return fail(IXB_ERR_INVALID, "K above 32768 could overflow the int32 product of uint8 x int4");
  if (!aligned16(a) || !aligned16(image) || !aligned16(out))
    return fail(IXB_ERR_INVALID, "u8i4 operands must be 16-byte aligned");
  GemmLaunch L;
  std::string err;
  if (plan_gemm(L, M, N, K, err, GEMM_B_W4)) return fail(IXB_ERR_INVALID, err);
  L.p.idesc = umma_idesc_u8s8(128, L.p.bn);
  L.p.out_kind = GEMM_OUT_I32;
  L.p.out32 = out;
  L.p.wq = image;
  L.p.eg = image + (uint64_t)N * (K / 2);
  if (encode_kmajor(&L.p.ta, a, M, K, 128, err)) return fail(IXB_ERR_CUDA, err);
  if (encode_w4(&L.p.tb, image, N, K, L.p.bn, err)) return fail(IXB_ERR_CUDA, err);
  return launch_gemm<GEMM_B_W4>(L, static_cast<cudaStream_t>(stream));
}

int ixb_w4a8_gemv(const int8_t* a, const uint8_t* image, const int32_t* shift, int8_t* out, int N, int K,
                  void* stream) {
  if (!a || !image || !shift || !out) return fail(IXB_ERR_INVALID, "null argument");
  if (int r = check_w4a8_shape(N, K)) return r;
  if (!aligned16(a) || !aligned16(image)) return fail(IXB_ERR_INVALID, "W4A8 operands must be 16-byte aligned");
  const uint8_t* eg = image + (uint64_t)N * (K / 2);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K <= 4 * 1024)  // at most four 16-byte loads per lane and column: two columns per warp
    IXB_CUDA(launch_dependent(w4a8_gemv_kernel<2>, dim3((unsigned)((N + 2 * kGemvWarps - 1) / (2 * kGemvWarps))),
                              dim3(kGemvThreads), 0, st, true, a, image, eg, shift, out, N, K));
  else
    IXB_CUDA(launch_dependent(w4a8_gemv_kernel<1>, dim3((unsigned)((N + kGemvWarps - 1) / kGemvWarps)), dim3(kGemvThreads),
                              0, st, true, a, image, eg, shift, out, N, K));
  return 0;
}

int ixb_gemm_plan_info(int M, int N, int K, int w4a8, int32_t* info, int n) {
  if (!info) return fail(IXB_ERR_INVALID, "null argument");
  GemmLaunch L;
  std::string err;
  if (plan_gemm(L, M, N, K, err, w4a8 ? GEMM_B_W4 : GEMM_B_TMA)) return fail(IXB_ERR_INVALID, err);
  const int32_t v[10] = {L.p.bn, L.p.mt, L.p.m_tiles, L.p.n_tiles, L.p.kblocks, L.p.stages, L.grid, L.smem,
                         L.p.tmem_cols, L.p.stage_bytes};
  for (int i = 0; i < n && i < 10; ++i) info[i] = v[i];
  return 0;
}

int ixb_decode_yolo(const ixb_decode_desc* d, const int8_t* egress, int batch, uint64_t egress_image_bytes,
                    const float* letterbox, int32_t capacity, float* boxes, float* scores, int32_t* classes,
                    int32_t* counts, void* stream) {
  if (!d || !egress || !letterbox || !boxes || !scores || !classes || !counts || batch < 1 || capacity < 0)
    return fail(IXB_ERR_INVALID, "bad decode arguments");
  if (reinterpret_cast<uintptr_t>(boxes) & 15) return fail(IXB_ERR_INVALID, "boxes must be 16-byte aligned");
  DecodeParams p;
  if (int r = prepare_decode(*d, egress_image_bytes, p)) return r;
  p.egress = egress;
  p.letterbox = letterbox;
  p.capacity = capacity;
  p.out_box = boxes;
  p.out_score = scores;
  p.out_class = classes;
  p.out_count = counts;
  return launch_decode(p, batch, static_cast<cudaStream_t>(stream));
}

// ixb_decode_yolo_noalloc: the decode with its table ranks and DFL checks in the library's own
// device array instead of memory the caller or a session allocates. For callers that may not
// allocate device memory at all: a plugin inside a host application that owns the CUDA context and
// its memory pool, or a loop whose timing cannot take cudaMalloc's implicit synchronisation.
}  // extern "C"

// 2 KB per GPU that loads the library, held until the process exits: the score ranks (uint16
// [768]) and the three DFL checks (int32 [3]) of one decode's tables. Host code must not hand this
// name to a kernel: on the host it is only the runtime's handle for the array, not its device
// address (noalloc_scratch looks that up).
constexpr int kNoAllocScratchBytes = 2048;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
static_assert(2 * kScoreVals + 3 * sizeof(int32_t) <= kNoAllocScratchBytes,
              "one table set's ranks and checks must fit the no-allocation scratch");

namespace {
// The scratch array's device address on the current device: looked up the first time a device
// asks, with that device current, then kept.
int noalloc_scratch(uint8_t** out) {
  static std::mutex mu;
  static uint8_t* addr[64] = {};
  int dev = 0;
  IXB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(IXB_ERR_UNSUPPORTED, "device index above 63");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* ptr = nullptr;
    IXB_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
    addr[dev] = static_cast<uint8_t*>(ptr);
  }
  *out = addr[dev];
  return 0;
}
}  // namespace

extern "C" {

int ixb_decode_yolo_noalloc(const ixb_decode_desc* d, const int8_t* egress, int batch, uint64_t egress_image_bytes,
                            const float* letterbox, int32_t capacity, float* boxes, float* scores, int32_t* classes,
                            int32_t* counts, void* stream) {
  if (!d || !egress || !letterbox || !boxes || !scores || !classes || !counts || batch < 1 || capacity < 0)
    return fail(IXB_ERR_INVALID, "bad decode arguments");
  if (reinterpret_cast<uintptr_t>(boxes) & 15) return fail(IXB_ERR_INVALID, "boxes must be 16-byte aligned");
  DecodeParams p;
  if (int r = prepare_decode(*d, egress_image_bytes, p)) return r;
  uint8_t* scratch = nullptr;
  if (int r = noalloc_scratch(&scratch)) return r;
  p.egress = egress;
  p.letterbox = letterbox;
  p.capacity = capacity;
  p.out_box = boxes;
  p.out_score = scores;
  p.out_class = classes;
  p.out_count = counts;
  // the tables kernel rewrites all 768 ranks and the three checks before the decode reads them, so
  // nothing from an earlier call carries over and nothing needs clearing
  uint16_t* ranks = reinterpret_cast<uint16_t*>(scratch);
  int32_t* toe = reinterpret_cast<int32_t*>(scratch + 2 * kScoreVals);
  p.ranks = ranks;
  p.toe = toe;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  decode_tables_kernel<<<1, kDecodeThreads, 0, st>>>(p, ranks, toe);
  IXB_CUDA(cudaGetLastError());
  return launch_decode(p, batch, st);
}

int ixb_decode_dense(const ixb_dense_head* heads, int32_t num_classes, const int8_t* egress, int batch,
                     uint64_t egress_image_bytes, float* out, void* stream) {
  if (!heads || !egress || !out || batch < 1 || batch > 65535) return fail(IXB_ERR_INVALID, "bad dense decode arguments");
  if (num_classes < 1 || num_classes > 1024) return fail(IXB_ERR_INVALID, "num_classes outside [1, 1024]");
  DenseParams p;
  memset(&p, 0, sizeof p);
  int total = 0;
  for (int h = 0; h < 3; ++h) {
    const ixb_dense_head& hd = heads[h];
    if (hd.grid < 1 || hd.grid > 4096 || !(hd.box_scale > 0.f) || !(hd.cls_scale > 0.f) || !(hd.stride > 0.f))
      return fail(IXB_ERR_INVALID, "dense decode head " + std::to_string(h) + ": bad grid, scale or stride");
    const uint64_t n = (uint64_t)hd.grid * hd.grid;
    if (hd.box_offset + 64 * n > egress_image_bytes || hd.cls_offset + (uint64_t)num_classes * n > egress_image_bytes)
      return fail(IXB_ERR_INVALID, "dense decode head " + std::to_string(h) + " outside the image's egress");
    DenseHeadDev& o = p.head[h];
    o.box_off = (long long)hd.box_offset;
    o.cls_off = (long long)hd.cls_offset;
    o.box_scale = hd.box_scale;
    o.box_zp = (float)hd.box_zero_point;
    o.cls_scale = hd.cls_scale;
    o.cls_zp = (float)hd.cls_zero_point;
    o.grid = hd.grid;
    o.anchors = (int)n;
    o.anchor_offset = total;
    o.stride = hd.stride;
    total += (int)n;
  }
  p.egress = egress;
  p.egress_image_bytes = (long long)egress_image_bytes;
  p.num_classes = num_classes;
  p.total_anchors = total;
  p.out = out;
  dense_decode_kernel<<<dim3((unsigned)((total + 255) / 256), (unsigned)batch), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(p);
  IXB_CUDA(cudaGetLastError());
  return 0;
}

int ixb_letterbox_frames(const uint8_t* frames, int batch, int src_w, int src_h, int src_stride, uint64_t frame_bytes,
                         const int8_t* lut, int8_t* out, int dst_w, int dst_h, int out_row_pixels,
                         uint64_t out_image_bytes, float* letterbox, void* stream) {
  if (!frames || !lut || !out || batch < 1 || src_w < 1 || src_h < 1 || dst_w < 1 || dst_h < 1)
    return fail(IXB_ERR_INVALID, "bad letterbox arguments");
  if (src_stride < 3 * src_w || frame_bytes < (uint64_t)src_stride * (src_h - 1) + 3ull * src_w ||
      out_row_pixels < dst_w || out_image_bytes < (uint64_t)out_row_pixels * 8 * (dst_h - 1) + 8ull * dst_w)
    return fail(IXB_ERR_INVALID, "letterbox strides smaller than the rows they hold");
  if (reinterpret_cast<uintptr_t>(out) & 7) return fail(IXB_ERR_INVALID, "letterbox output must be 8-byte aligned");
  // the reference's float32 letterbox geometry (preprocess_simd.c:352-363)
  const float scale_w = (float)dst_w / (float)src_w, scale_h = (float)dst_h / (float)src_h;
  const float scale = scale_w < scale_h ? scale_w : scale_h;
  int nw = (int)std::floor((float)src_w * scale + 0.5f), nh = (int)std::floor((float)src_h * scale + 0.5f);
  if (nw > dst_w) nw = dst_w;
  if (nh > dst_h) nh = dst_h;
  if (nw < 1 || nh < 1) return fail(IXB_ERR_INVALID, "letterboxed image is empty");
  LetterboxParams p;
  memset(&p, 0, sizeof p);
  p.frames = frames;
  p.frame_bytes = (long long)frame_bytes;
  p.src_w = src_w;
  p.src_h = src_h;
  p.src_stride = src_stride;
  p.dst_w = dst_w;
  p.dst_h = dst_h;
  p.nw = nw;
  p.nh = nh;
  p.pad_top = (dst_h - nh) / 2;
  p.pad_left = (dst_w - nw) / 2;
  p.fx = (float)src_w / (float)nw;
  p.fy = (float)src_h / (float)nh;
  p.lut = lut;
  p.out = out;
  p.out_row_pixels = out_row_pixels;
  p.out_image_bytes = (long long)out_image_bytes;
  p.batch = batch;
  if (letterbox) {
    letterbox[0] = (float)p.pad_top;
    letterbox[1] = (float)p.pad_left;
    letterbox[2] = scale;
  }
  const long long total = (long long)batch * dst_h * dst_w;
  const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 16);
  letterbox_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  IXB_CUDA(cudaGetLastError());
  return 0;
}

int ixb_session_letterbox(ixb_session* s, const uint8_t* frames, int batch, int src_w, int src_h, int src_stride,
                          uint64_t frame_bytes, float* letterbox) {
  if (!s) return fail(IXB_ERR_INVALID, "null session");
  if (batch < 1 || batch > s->plan.max_batch) return fail(IXB_ERR_INVALID, "batch outside [1, max_batch]");
  if (s->pending || s->any_busy()) return fail(IXB_ERR_INVALID, "runs are still in flight");
  IXB_CUDA(cudaSetDevice(s->device));
  const ixb_plan& pl = s->plan;
  const int row = pl.img_w + 4;
  int8_t* base = reinterpret_cast<int8_t*>(s->arena + pl.input.offset) + ((long long)row + 1) * 8;
  if (int r = ixb_letterbox_frames(frames, batch, src_w, src_h, src_stride, frame_bytes,
                                   reinterpret_cast<const int8_t*>(s->arena + pl.input_lut_offset), base, pl.img_w,
                                   pl.img_h, row, (uint64_t)(pl.img_h + 2) * row * 8, letterbox, s->stream))
    return r;
  // a stem over the space-to-depth view reads the letterboxed image repacked into that view
  if (pl.input_s2d)
    return launch_ingress_s2d(nullptr, reinterpret_cast<const int8_t*>(s->arena + pl.input.offset), nullptr, batch,
                              pl.img_h, pl.img_w, s->arena, pl.input_s2d_view, s->stream);
  return 0;
}

int ixb_quantize_images(const uint8_t* images, const int8_t* lut, int batch, int h, int w, int8_t* padded_nhwc4,
                        void* stream) {
  if (!images || !lut || !padded_nhwc4 || batch < 1 || h < 1 || w < 4) return fail(IXB_ERR_INVALID, "bad arguments");
  return launch_quantize(images, lut, batch, h, w, padded_nhwc4, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
