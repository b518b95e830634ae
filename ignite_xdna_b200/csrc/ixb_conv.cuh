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
// Storage: one plane per 16-channel chunk, [batch][H+2][W+2] pixels of 16 bytes with a zero
// halo ring per image and zero guard pixels around the plane; plane strides are whole images,
// so a tensor map can address chunk c, image n as image c * (plane / image) + n. A K-chunk of
// 128 output pixels is then 128 rows of 16 bytes, a column of UMMA core matrices in smem.
//
// GEMM view: M = output pixels, N = output channels (n_tile per CTA, one TMEM column each),
// K = input channels x taps in 32-byte MMA steps. A tile is MT blocks of 128 pixels; block b
// accumulates into TMEM columns [b * n_tile, (b+1) * n_tile). A-operand producers by mode:
//  * WINDOW (stride 1, same resolution): the tile is 128*MT consecutive pixels of the flattened
//    padded image; tap (ky, kx) of output pixel m reads padded pixel m + (ky-1)(W+2) + (kx-1), so
//    ONE window of 128*MT + 2((W+2)+1) pixels per chunk feeds all nine taps, each tap the same smem
//    window through a descriptor whose start moves 16 bytes per pixel of shift. A window is one
//    bulk copy (TMA engine) per chunk. Halo outputs are computed and dropped.
//  * IM2COL (3x3 stride 2): the tile is 128*MT output pixels (one spare column per output row); per
//    (image row ky, kx in {0, 1}, chunk) one TMA im2col load walks the filter positions (element
//    stride 2 on the padded plane) and lands the tile's rows (+ 8) for that tap; kx = 2 of output x
//    is kx = 0 of output x + 1, read as that slot one row on.
//  * STEM: the image stored as 8-byte pixels (3 channels + 5 zero) and read as 16-byte pixel pairs;
//    output pixel (y, x) tap (ky, pair p) is the pair at padded row 2y+ky, column 2x+2p. Pair p = 1
//    of output x is pair 0 of output x + 1, so one TMA im2col load per image row ky (tile + 8 rows)
//    serves both pairs, the second as the same slot one row on; the M space carries one spare output
//    column per row (computed, then dropped) so that shift never crosses into the next output row.
//  * GATHER (a 1x1 conv over a concat that includes a nearest-2x upsampled view): per-row 16-byte
//    cp.async gathers by 128 producer threads from a per-tile table of output coordinates.
// Shared-memory operands use the K-major no-swizzle core-matrix layout: A as [slot][pixel][16 B]
// (SBO 128 B), B as [n/8][K-half][8][16 B] (SBO 256 B, LBO 128 B), prepacked on the host in the
// schedule's order. Each MMA's A descriptor carries its own start and LBO: the two 32-byte K-halves
// are two A slots (two chunks of one tap, or one chunk at two taps).
//
// The kernel is persistent and warp-specialised:
//   epilogue warps (16, or 8 for GATHER): TMEM -> registers -> epilogue -> global; warp w reads
//            TMEM lane quarter w % 4, the warpgroups take shares of the tile's (block, 16-column)
//            units
//   producer: one thread issuing bulk / TMA copies (4 warps of cp.async for GATHER)
//   MMA warps (3, or 4 for GATHER): each issues its share of each K-block's MMAs from one elected
//            lane (a single issuing thread reaches only ~95 cycles per MMA)
// Several TMEM accumulators (two for the widest tiles, up to eight for narrow ones) let the
// epilogue of one tile overlap the MMAs of the next ones and absorb the jitter between the two
// sides. When a CTA's weights fit, they are loaded once and stay resident in shared memory.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ixb_ptx.cuh"
#include "../../include/ixb200.h"

namespace ixb {

struct SegDev {
  const int8_t* base;  // padded pixel 0 of image 0 in the view's first chunk plane
  long long plane;     // bytes between chunk planes
  int chunk_begin, chunks;  // 16-channel chunks of the logical input this view supplies
  int H, W, up2, P;         // stored size, upsampled view, padded pixels per image
  int plane_images;         // plane stride in images
};

// One K-block: its A slots (slot s holds chunk chunk0 + s / ntaps at tap tap0 + s % ntaps; for
// WINDOW ntaps = 1 and the taps live in the MMA ops as window shifts), its MMAs (op0 .. op0+nops-1
// of the op table) and its weights.
struct KBlockDev {
  int b_off, b_bytes;
  int16_t op0, nops, chunk0, nchunks, tap0, ntaps;
};
constexpr int kMaxKBlocks = 96;
constexpr int kMaxOps = 160;
constexpr int kMaxAcc = 8;

// GATHER: one input chunk as the producer reads it, from a shared-memory table filled at start
// (a dynamically indexed read of the kernel parameters' segment table costs hundreds of cycles).
struct GatherChunk {
  const int8_t* base;  // the chunk's plane: padded pixel 0 of image 0
  int P, W2, up2, pad;  // padded pixels per image, padded width, nearest-2x upsampled view
};


struct ConvParams {
  alignas(64) CUtensorMap tmap;  // TMA im2col map (IM2COL, STEM)
  int mode, k, stride, pad;
  int H, W, Ho, Wo, batch;
  int m_total;
  int cin_chunks, cp, kblocks;
  int mt, tile_rows, m_tiles;
  int rowsA, win_origin;
  int a_stage_bytes, b_block_bytes, stage_bytes, stages;
  int b_resident, a_off, tbl_off, bar_off, bias_off;
  int ctab_off;  // per input chunk: WINDOW its plane's address, GATHER its GatherChunk (shared memory)
  int n_tile, acc_cols, tmem_cols, issuers;  // MMA issuing warps
  int nacc;                                  // TMEM accumulators (2 .. kMaxAcc) of acc_cols columns
  int ew;                                           // epilogue warps (8 or 16)
  uint32_t idesc;
  int nseg;
  SegDev seg[IXB_MAX_SEGS];
  const uint8_t* wpack;
  long long w_ntile_stride;
  const int32_t* bias;
  const int8_t* lut;
  int shift;      // SRS shift of the float path, at most 16 (negative: a left shift)
  int pre_shift;  // shift - 16 when the layer's shift exceeds 16: an exact sticky pre-reduction first
  int has_res;
  SegDev res;
  int res_lsh_m, res_lsh_r, res_shift;
  int out_nchw;
  SegDev out;
  int out2_kind;  // IXB_OUT2_*: a second copy (2x2-upsampled or space-to-depth), or only the latter
  SegDev out2;
  int8_t* egress;
  long long egress_img;
  int egress_ch;  // channels the head writes (the rest of cout are zero-weight padding)
  int cout;
  FastDiv fd_P, fd_W2, fd_hw, fd_Wo;  // padded pixels per image, padded width, Ho*Wm, Wm
  int Wm;                             // output row length in M space: Wo, or Wo + 1 for STEM
  unsigned long long* stats;          // optional per-CTA role counters (kStatWords per CTA), or null
  unsigned long long* trace;          // optional launch timeline (globaltimer ns), or null: see trace_mark
  KBlockDev kb[kMaxKBlocks];          // the K schedule
  uint32_t op_a[kMaxOps];             // per MMA: A start (16-byte units from the stage) | LBO (16-byte units) << 16
  uint16_t op_b[kMaxOps];             // per MMA: B start (16-byte units from the K-block's weights)
};

// Per-CTA role counters (clock64 cycles) written when ConvParams::stats is set.
enum : int {
  kStatEpiWait = 0,   // epilogue warp 0 waiting for an accumulator
  kStatEpiWork,       // epilogue warp 0 draining accumulators
  kStatMmaWaitFull,   // MMA issuer 0 waiting for loaded stages
  kStatMmaWaitAcc,    // MMA issuer 0 waiting for a free accumulator
  kStatMmaIssue,      // MMA issuer 0 issuing
  kStatProdWait,      // producer 0 waiting for free stages
  kStatProdWork,      // producer 0 issuing loads
  kStatTotal,         // CTA lifetime
  kStatTiles,
  kStatWords = 16
};

constexpr int kBlockM = 128;
// Warp layout per (mode, epilogue warps EW): EW epilogue warps, the producer warps, then the MMA
// warps (a warp issues an MMA only every ~95 cycles, so several issue).
//   EW = 16: 16 epilogue + 1 producer + 3 MMA (WINDOW, IM2COL, STEM): 20 warps at 96 registers.
//            The drain is latency-bound (dependent conversions, TMEM and table loads), so four
//            epilogue warps per SM sub-partition instead of three took the v8n step from 1.158 to
//            1.127 ms with no spills.
//   EW = 8:   8 epilogue + 4 producer + 4 MMA (GATHER): 16 warps at 128 registers.
__host__ __device__ constexpr int prod_warps(int mode) { return mode == IXB_MODE_GATHER ? 4 : 1; }
__host__ __device__ constexpr int mma_warp0(int mode, int ew) { return ew + prod_warps(mode); }
__host__ __device__ constexpr int mma_warps(int ew) { return ew == 8 ? 4 : 3; }
__host__ __device__ constexpr int conv_threads(int mode, int ew) { return 32 * (mma_warp0(mode, ew) + mma_warps(ew)); }
constexpr int kGatherThreads = 128;

__device__ __forceinline__ void producer_bar_sync() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

__device__ __forceinline__ int seg_of_chunk(const ConvParams& p, int gc) {
  int si = -1;
#pragma unroll
  for (int s = 0; s < IXB_MAX_SEGS; ++s)
    if (s < p.nseg && gc >= p.seg[s].chunk_begin && gc < p.seg[s].chunk_begin + p.seg[s].chunks) si = s;
  return si;
}

// TMA im2col load of the map's pixelsPerColumn rows, 16 bytes each, completing on bar.
__device__ __forceinline__ void tma_im2col(void* dst, const CUtensorMap* tm, int w, int h, int n, int off_w, int off_h,
                                           uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(0), "r"(w), "r"(h), "r"(n), "r"(smem_u32(bar)), "h"((uint16_t)off_w), "h"((uint16_t)off_h)
      : "memory");
}

// Launch timeline, when ConvParams::trace is set: word 0 = earliest CTA start, word 1 = earliest
// time a CTA's producer was past the wait for the previous kernel (its inputs were ready),
// word 2 = latest CTA end. Words 0 and 1 start at ~0, word 2 at 0.
__device__ __forceinline__ void trace_mark(unsigned long long* tr, int word) {
  if (!tr) return;
  const unsigned long long t = global_ns();
  if (word < 2) atomicMin(tr + word, t);
  else atomicMax(tr + word, t);
}

__device__ __forceinline__ void write_stats(const ConvParams& p, int idx, unsigned long long v) {
  if (p.stats) p.stats[(blockIdx.y * gridDim.x + blockIdx.x) * kStatWords + idx] = v;
}

// ---------------------------------------------------------------- producers
// One thread: bulk (WINDOW) or TMA im2col (IM2COL, STEM) copies per K-block, plus streamed weights.
template <int MODE>
__device__ __forceinline__ void produce_single(const ConvParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                               int ntile) {
  const int S = p.stages;
  const uint32_t slot_bytes = (uint32_t)p.rowsA * 16;
  int stage = 0;
  uint32_t ph = 0;
  long long tw = 0, tk = 0;
  for (int t = blockIdx.x; t < p.m_tiles; t += gridDim.x) {
    const int m0 = t * p.tile_rows;
    const long long wb = (long long)m0 - p.win_origin;
    int img0 = 0, y0 = 0, x0 = 0;
    if (MODE != IXB_MODE_WINDOW) {
      img0 = (int)fdiv((uint32_t)m0, p.fd_hw);
      const int rem = m0 - img0 * (int)p.fd_hw.d;
      y0 = (int)fdiv((uint32_t)rem, p.fd_Wo);
      x0 = rem - y0 * p.Wm;
    }
    for (int kb = 0; kb < p.kblocks; ++kb) {
      const long long c0 = clock64();
      mbar_wait(&empty[stage], ph ^ 1);
      const long long c1 = clock64();
      tw += c1 - c0;
      uint8_t* As = smem + p.a_off + stage * p.stage_bytes;
      const KBlockDev K = p.kb[kb];  // one read of the K-block's entry per K-block
      const int nslots = K.nchunks * K.ntaps;
      mbar_arrive_expect_tx(&full[stage], (uint32_t)nslots * slot_bytes + (p.b_resident ? 0u : (uint32_t)K.b_bytes));
      if (MODE == IXB_MODE_WINDOW) {
        // one slot per chunk (the taps are window shifts); the chunk's plane comes from the
        // shared-memory table (a dynamically indexed read of the kernel parameters costs a few
        // hundred cycles per copy)
        const int8_t* const* ctab = reinterpret_cast<const int8_t* const*>(smem + p.ctab_off);
        for (int sl = 0; sl < nslots; ++sl)
          bulk_g2s(As + sl * slot_bytes, ctab[K.chunk0 + sl] + wb * 16, slot_bytes, &full[stage]);
      } else {
        for (int sl = 0; sl < nslots; ++sl) {
          const int gc = K.chunk0 + sl / K.ntaps;
          const int tap = K.tap0 + sl % K.ntaps;
          if (MODE == IXB_MODE_IM2COL) {  // loaded tap = 2 ky + kx, kx in {0, 1}
            const SegDev& s = p.seg[0];
            tma_im2col(As + sl * slot_bytes, &p.tmap, 2 * x0, 2 * y0, (gc - s.chunk_begin) * s.plane_images + img0,
                       tap & 1, tap >> 1, &full[stage]);
          } else {  // STEM: slot = image row ky; pair 1 of output x is pair 0 of x + 1, one row on
            tma_im2col(As + sl * slot_bytes, &p.tmap, x0, 2 * y0, img0, 0, tap, &full[stage]);
          }
        }
      }
      if (!p.b_resident)
        bulk_g2s(As + p.a_stage_bytes, p.wpack + ntile * p.w_ntile_stride + K.b_off, K.b_bytes, &full[stage]);
      tk += clock64() - c1;
      if (++stage == S) {
        stage = 0;
        ph ^= 1;
      }
    }
  }
  write_stats(p, kStatProdWait, tw);
  write_stats(p, kStatProdWork, tk);
}

// 128 threads: 16-byte cp.async row gathers (a concat including an upsampled view).
__device__ __forceinline__ void produce_gather(const ConvParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                               int ntile, int ptid) {
  const int nch = 2 * p.cp;
  const int c = ptid % nch;  // 128 is a multiple of nch, so each thread keeps one slot
  const int step = kGatherThreads / nch;
  const int S = p.stages;
  const int hw = p.Ho * p.Wo;
  // Per tile, one row table entry per output pixel: {image, y, x}; image -1 marks rows past the batch.
  int4* tbl = reinterpret_cast<int4*>(smem + p.tbl_off);
  const GatherChunk* gtab = reinterpret_cast<const GatherChunk*>(smem + p.ctab_off);
  long long tw = 0;
  const long long cstart = clock64();
  int stage = 0;
  uint32_t ph = 0;
  int it = 0;
  for (int t = blockIdx.x; t < p.m_tiles; t += gridDim.x, ++it) {
    const int m0 = t * p.tile_rows;
    int4* T = tbl + (it & 1) * p.tile_rows;
    for (int r = ptid; r < p.tile_rows; r += kGatherThreads) {
      const int m = m0 + r;
      if (m < p.m_total) {
        const int img = (int)fdiv((uint32_t)m, p.fd_hw);
        const int rem = m - img * hw;
        const int y = (int)fdiv((uint32_t)rem, p.fd_Wo);
        T[r] = make_int4(img, y, rem - y * p.Wo, 0);
      } else {
        T[r] = make_int4(-1, 0, 0, 0);
      }
    }
    producer_bar_sync();
    for (int kb = 0; kb < p.kblocks; ++kb) {
      const long long c0 = clock64();
      mbar_wait(&empty[stage], ph ^ 1);
      tw += clock64() - c0;
      uint8_t* dst = smem + p.a_off + stage * p.stage_bytes + c * p.rowsA * 16;
      const KBlockDev K = p.kb[kb];  // one read per K-block
      if (c < K.nchunks) {
        const GatherChunk g = gtab[K.chunk0 + c];
        for (int r = ptid / nch; r < p.tile_rows; r += step) {
          const int4 e = T[r];
          if (e.x >= 0) {
            const int iy = g.up2 ? (e.y >> 1) : e.y, ix = g.up2 ? (e.z >> 1) : e.z;
            cp_async16(dst + r * 16, g.base + ((long long)e.x * g.P + (iy + 1) * g.W2 + (ix + 1)) * 16, 16u);
          } else {
            cp_async16(dst + r * 16, g.base, 0u);
          }
        }
      }
      cp_async_mbar_arrive(&full[stage]);
      if (!p.b_resident && ptid == 0) {
        mbar_arrive_expect_tx(&full[stage], K.b_bytes);
        bulk_g2s(smem + p.a_off + stage * p.stage_bytes + p.a_stage_bytes, p.wpack + ntile * p.w_ntile_stride + K.b_off,
                 K.b_bytes, &full[stage]);
      }
      if (++stage == S) {
        stage = 0;
        ph ^= 1;
      }
    }
  }
  if (ptid == 0) {
    write_stats(p, kStatProdWait, tw);
    write_stats(p, kStatProdWork, clock64() - cstart - tw);
  }
}

// ---------------------------------------------------------------- MMA issuer
// The accumulators start at the bias (the epilogue resets each one after draining it, and the
// kernel sets them all at start), so every MMA accumulates and a K-block's MMAs can be issued by
// several threads in any order. A K-block's MMAs are its items (op o, 128-row block b), numbered
// i = (o - op0) * mt + b; issuer `who` of p.issuers takes the items with i % issuers == who, so the
// issuers share the work evenly even when a K-block has fewer ops than issuers (1x1 layers). One
// thread issues an MMA only every ~95 cycles; an M=128, K=32 MMA occupies the tensor core for ~39
// cycles at N <= 32 (its A and B operands read from shared memory), 48 at N = 64, 64 at N = 128,
// so three issuers keep it fed. Every issuer commits every stage, so a stage is released when all
// of its MMAs are done.
// Each issuer is a whole warp: the loop runs on all 32 lanes from a warp index made uniform by a
// shuffle, so the op-table reads and the descriptors live in uniform registers, and one elected
// lane issues each MMA and commit (a single-lane branch measured ~2.5 % slower over a whole step).
template <int MODE>
__device__ __forceinline__ void issue_mma(const ConvParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty,
                                          uint64_t* acc_full, uint64_t* acc_empty, uint64_t* bres_bar, uint32_t tmem,
                                          int who) {
  if (p.b_resident) mbar_wait(bres_bar, 0);
  const int S = p.stages, I = p.issuers, NA = p.nacc;
  int stage = 0, acc = 0;
  uint32_t ph = 0, aph = 0;
  uint32_t wf = 0, wa = 0, wi = 0;  // role cycles (32-bit: a launch lasts far less than 2^32 cycles)
  // A: SBO 128 B, sm_100 descriptor; blocks are 128 rows (128 16-byte units) apart in a stage
  const uint64_t a_hi = ((uint64_t)(128 >> 4) << 32) | ((uint64_t)1 << 46);
  const uint32_t a_base = smem_u32(smem + p.a_off) >> 4;
  const uint32_t w_base = smem_u32(smem);
  const int mt_lg = __ffs(p.mt) - 1;  // mt is a power of two, 1 .. 16
  for (int t = blockIdx.x; t < p.m_tiles; t += gridDim.x) {
    uint32_t c0 = (uint32_t)clock();
    mbar_wait(&acc_empty[acc], aph ^ 1);
    uint32_t c1 = (uint32_t)clock();
    wa += c1 - c0;
    tc_fence_after();
    const uint32_t d_acc = tmem + acc * p.acc_cols;
    for (int kb = 0; kb < p.kblocks; ++kb) {
      c0 = (uint32_t)clock();
      mbar_wait(&full[stage], ph);
      c1 = (uint32_t)clock();
      wf += c1 - c0;
      if (MODE == IXB_MODE_GATHER) fence_proxy_async_smem();  // cp.async (generic proxy) writes -> UMMA reads
      tc_fence_after();
      // A descriptor = stage base + op start / LBO (16-byte units) + block; B = K-block weights
      // + op start. Additions to the low 14-bit address field cannot carry (smem < 256 KB). The
      // op table is read from the kernel parameters with warp-uniform indices, so the descriptors
      // stay in uniform registers, which tcgen05.mma takes its operands from.
      const KBlockDev& K = p.kb[kb];
      const uint32_t a0 = a_base + (uint32_t)((stage * p.stage_bytes) >> 4);
      const uint32_t b0 = p.b_resident ? w_base + K.b_off : ((a_base << 4) + stage * p.stage_bytes + p.a_stage_bytes);
      const uint64_t bdesc0 = umma_desc(b0, 128, 256);
      const int items = (int)K.nops << mt_lg;
#pragma unroll 2
      for (int i = who; i < items; i += I) {
        const int o = K.op0 + (i >> mt_lg), b = i & (p.mt - 1);
        const uint32_t opa = p.op_a[o];
        const uint64_t ad = a_hi | (uint64_t)((a0 + (opa & 0xFFFFu)) | ((opa >> 16) << 16));
        const uint64_t bd = bdesc0 + p.op_b[o];
        if (elect_one())
          umma_s8(d_acc + (uint32_t)(b * p.n_tile), ad + (uint64_t)(b * ((kBlockM * 16) >> 4)), bd, p.idesc, 1u);
        __syncwarp();
      }
      if (elect_one()) umma_commit(&empty[stage]);
      __syncwarp();
      wi += (uint32_t)clock() - c1;
      if (++stage == S) {
        stage = 0;
        ph ^= 1;
      }
    }
    if (elect_one()) umma_commit(&acc_full[acc]);
    __syncwarp();
    if (++acc == NA) {
      acc = 0;
      aph ^= 1;
    }
  }
  if (who == 0 && (threadIdx.x & 31) == 0) {
    write_stats(p, kStatMmaWaitFull, wf);
    write_stats(p, kStatMmaWaitAcc, wa);
    write_stats(p, kStatMmaIssue, wi);
  }
}

// ---------------------------------------------------------------- epilogue
// 16 accumulators of one row (bias included) -> 16 int8 outputs: RNE shift and int8 clamp (one
// float conversion), table, residual.
// `lut` points at entry 128 of the 256-byte table (static shared memory), so it is indexed by the
// clamped value directly; the bytes are gathered into words with byte permutes.
// Shift-round-saturate through the float unit: sat_s8(rne(c / 2^s)) as f = float(c) (round to
// nearest), f * 2^-s (exact: a power of two, no overflow or underflow for s in [0, 16]), then a
// float -> s8 conversion that rounds to nearest even and saturates. Exact for every int32 c: for
// |c| < 2^24 float(c) == c, and for |c| >= 2^24 both |c / 2^s| and |f * 2^-s| are >= 256, so the
// exact and the float path saturate to the same end. Three instructions (plus a sign extension
// of the byte) where the integer form takes seven; the epilogue's arithmetic bounds most layers.
// A negative s (a left shift) is exact the same way: f * 2^|s| is c * 2^|s| for |c| < 2^24 and
// saturates otherwise. Shifts above 16 go through pre_reduce first (the generic drain).
__device__ __forceinline__ float pow2_neg(int s) { return __int_as_float((127 - s) << 23); }
__device__ __forceinline__ int srs_s8(int c, float scale) {
  const float f = __int2float_rn(c) * scale;
  int r;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(f));
  return (int)(int8_t)r;  // the s8 result, sign-extended whatever the register's upper bits hold
}

// acc / 2^k rounded to nearest even equals rne(c' / 2^16) for c' = (acc >> k) with the dropped
// bits or'ed into bit 0 (a sticky bit below the rounding position): the float path then covers
// SRS shifts of 16 + k exactly, whatever the accumulator's magnitude.
__device__ __forceinline__ uint32_t pre_reduce(uint32_t v, int k) {
  const int c = (int)v;  // k in [1, 31]
  return (uint32_t)(c >> k) | ((v & ((1u << k) - 1u)) != 0u ? 1u : 0u);
}

// A linear layer (identity table, the detect heads): the same rounding, the int8 saturation done by
// the packing conversion, two of which pack four values (no table lookups, no byte permutes).
__device__ __forceinline__ uint32_t pack_sat_s8(int r0, int r1, int r2, int r3) {
  uint32_t hi, w;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(r3), "r"(r2), "r"(0u));  // bytes {r2, r3}
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(r1), "r"(r0), "r"(hi));  // {r0, r1, r2, r3}
  return w;
}
__device__ __forceinline__ uint4 epilogue16_linear(const uint32_t (&v)[16], float scale) {
  int r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = __float2int_rn(__int2float_rn((int)v[i]) * scale);
  return make_uint4(pack_sat_s8(r[0], r[1], r[2], r[3]), pack_sat_s8(r[4], r[5], r[6], r[7]),
                    pack_sat_s8(r[8], r[9], r[10], r[11]), pack_sat_s8(r[12], r[13], r[14], r[15]));
}

// The table index t1 + 128 of t1 = clamp(rne(c * 2^-s), -128, 127) in one conversion: rne(x) + 128 =
// rne(x + 128) (128 is even). For s <= 16 the fma computing x + 128 = float(c) * 2^-s + 128 is
// exact whenever |x + 128| < 256 (x's fraction is a multiple of 2^-16; a left shift gives an
// integer), and beyond that both forms saturate (as in srs_s8, float(c) is exact below 2^24); the
// unsigned saturating conversion clamps to [0, 255]. It saves the s8 form's sign extension (1.4 %
// of a step).
__device__ __forceinline__ uint32_t srs_index(int c, float scale) {
  uint32_t r;
  asm("cvt.rni.sat.u8.f32 %0, %1;" : "=r"(r) : "f"(fmaf(__int2float_rn(c), scale, 128.f)));
  return r;
}

template <bool RES>
__device__ __forceinline__ uint4 epilogue16(const uint32_t (&v)[16], const uint8_t* lut, float scale,
                                            const ConvParams& p, float rscale, uint4 r4) {
  uint32_t t[16];
  const int8_t* rv = reinterpret_cast<const int8_t*>(&r4);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    // the accumulator started at the bias: t1 = clamp(rne(acc >> shift)), then the table
    uint32_t u = (lut - 128)[srs_index((int)v[i], scale)];
    if (RES) {
      const int y = ((int)(int8_t)u << p.res_lsh_m) + ((int)rv[i] << p.res_lsh_r);  // |y| < 2^24
      u = (uint32_t)(uint8_t)srs_s8(y, rscale);
    }
    t[i] = u;
  }
  uint4 o;
  o.x = __byte_perm(__byte_perm(t[0], t[1], 0x0040), __byte_perm(t[2], t[3], 0x0040), 0x5410);
  o.y = __byte_perm(__byte_perm(t[4], t[5], 0x0040), __byte_perm(t[6], t[7], 0x0040), 0x5410);
  o.z = __byte_perm(__byte_perm(t[8], t[9], 0x0040), __byte_perm(t[10], t[11], 0x0040), 0x5410);
  o.w = __byte_perm(__byte_perm(t[12], t[13], 0x0040), __byte_perm(t[14], t[15], 0x0040), 0x5410);
  return o;
}

struct RowInfo {
  int opix, img, oy, ox;
  bool valid;
};

template <int MODE>
__device__ __forceinline__ RowInfo decode_row(const ConvParams& p, int m) {
  RowInfo r;
  r.valid = m < p.m_total;
  if (MODE == IXB_MODE_WINDOW) {
    r.img = (int)fdiv((uint32_t)m, p.fd_P);
    const int rem = m - r.img * (int)p.fd_P.d;
    const int yp = (int)fdiv((uint32_t)rem, p.fd_W2), xp = rem - yp * (p.W + 2);
    r.valid = r.valid && yp >= 1 && yp <= p.H && xp >= 1 && xp <= p.W;
    r.opix = m;
    r.oy = yp - 1;
    r.ox = xp - 1;
  } else {
    r.img = (int)fdiv((uint32_t)m, p.fd_hw);
    const int rem = m - r.img * (int)p.fd_hw.d;
    r.oy = (int)fdiv((uint32_t)rem, p.fd_Wo);
    r.ox = rem - r.oy * p.Wm;
    r.valid = r.valid && r.ox < p.Wo;  // STEM computes one spare column per output row
    r.opix = r.img * (p.Ho + 2) * (p.Wo + 2) + (r.oy + 1) * (p.Wo + 2) + (r.ox + 1);
  }
  return r;
}

// The residual's 16 bytes for (row, output chunk of n-tile `ntile`, chunk jj), loaded ahead of use.
__device__ __forceinline__ uint4 residual_load(const ConvParams& p, const RowInfo& r, int ntile, int jj) {
  if (!p.has_res || !r.valid) return make_uint4(0, 0, 0, 0);
  const int oc = ntile * (p.n_tile >> 4) + jj;
  return *reinterpret_cast<const uint4*>(p.res.base + (long long)oc * p.res.plane + (long long)r.opix * 16);
}

__device__ __forceinline__ void store_piece(const ConvParams& p, const RowInfo& r, int ntile, int jj, const uint32_t (&v)[16],
                                            uint4 r4, const uint8_t* lut_s, float scale, float rscale,
                                            bool linear) {
  const int nj = p.n_tile / 16;
  const int oc = ntile * nj + jj;  // output chunk
  uint4 o;
  if (linear && !p.has_res) {
    o = epilogue16_linear(v, scale);
  } else if (p.has_res) {
    o = epilogue16<true>(v, lut_s, scale, p, rscale, r4);
  } else {
    o = epilogue16<false>(v, lut_s, scale, p, rscale, make_uint4(0, 0, 0, 0));
  }
  if (!p.out_nchw) {
    if (p.out2_kind != IXB_OUT2_S2D_ONLY)
      *reinterpret_cast<uint4*>(const_cast<int8_t*>(p.out.base) + (long long)oc * p.out.plane + (long long)r.opix * 16) = o;
    if (p.out2_kind >= IXB_OUT2_S2D) {  // pixel (y, x), chunk oc -> (y/2, x/2), chunk phase * chunks + oc
      const int ph = (r.oy & 1) * 2 + (r.ox & 1);
      *reinterpret_cast<uint4*>(const_cast<int8_t*>(p.out2.base) + (long long)(ph * (p.cout >> 4) + oc) * p.out2.plane +
                                ((long long)r.img * p.out2.P + (long long)((r.oy >> 1) + 1) * (p.out2.W + 2) +
                                 (r.ox >> 1) + 1) * 16) = o;
    } else if (p.out2_kind == IXB_OUT2_UP2) {  // pixel (y, x) -> (2y + dy, 2x + dx) of the upsampled copy
      const int W2 = p.out2.W + 2;
      uint4* u = reinterpret_cast<uint4*>(const_cast<int8_t*>(p.out2.base) + (long long)oc * p.out2.plane +
                                          ((long long)r.img * p.out2.P + (long long)(2 * r.oy + 1) * W2 + 2 * r.ox + 1) * 16);
      u[0] = o;
      u[1] = o;
      u[W2] = o;
      u[W2 + 1] = o;
    }
  } else {
    int8_t* e = p.egress + (long long)r.img * p.egress_img + r.oy * p.Wo + r.ox;
    const long long plane = (long long)p.Ho * p.Wo;
    const int8_t* ob = reinterpret_cast<const int8_t*>(&o);
    const int c0 = ntile * p.n_tile + jj * 16;
    if (c0 + 16 <= p.egress_ch) {
#pragma unroll
      for (int i = 0; i < 16; ++i) e[(c0 + i) * plane] = ob[i];
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (c0 + i < p.egress_ch) e[(c0 + i) * plane] = ob[i];
    }
  }
}

// Drain one accumulator: warp w reads TMEM lane quarter w % 4. The tile's units (128-row block,
// 16-column chunk), in block-major order, are split into one contiguous share per warpgroup, so a
// thread decodes its row once per block. One unit at a time (16 accumulators in registers): two
// units in flight measured slower, the extra registers cost the arithmetic its interleaving. Which
// warpgroup takes which share rotates with the CTA's tile count `it`: when the units do not divide
// evenly (4 units over 3 warpgroups), each warpgroup takes the larger share in turn instead of one
// always lagging. A drained unit is set back to the bias, the value the next tile's accumulation
// starts from.
// KIND picks the layer's epilogue once per kernel, so that the hot loop holds only its own path:
// with every path inlined in one loop (table, linear, residual, NCHW head) the 1x1 layers measured
// ~20 % slower.
enum : int { kEpiTable = 0, kEpiLinear = 1, kEpiResidual = 2, kEpiGeneric = 3, kEpiTableS2D = 4, kEpiLinearNCHW = 5 };
template <int MODE, int EW, int KIND>
__device__ __forceinline__ void conv_epilogue_tile(const ConvParams& p, uint32_t tacc, int m0, int ntile, int warp,
                                                   int lane, const uint8_t* lut_s, const int4* bias4_s, int it,
                                                   bool linear) {
  constexpr int NG = EW / 4;
  const int q = warp & 3, g = ((warp >> 2) + it) % NG;
  const int nj = p.n_tile >> 4;
  const float scale = pow2_neg(p.shift), rscale = pow2_neg(p.res_shift);
  const uint32_t lane_base = tacc + ((uint32_t)(q * 32) << 16);
  const int units = p.mt * nj;
  const int u_end = ((g + 1) * units) / NG;
  int u = (g * units) / NG;
  // (b, j) of unit u without a division: walk from the share's start
  int b = 0, j = u;
  while (j >= nj) {
    j -= nj;
    ++b;
  }
  const int row_in_block = q * 32 + lane;
  int decoded_b = -1;
  RowInfo r{};
  for (; u < u_end; ++u) {
    uint32_t v[16];
    const uint32_t c = lane_base + (uint32_t)(b * p.n_tile + j * 16);
    tmem_ld16(c, v);
    if (b != decoded_b) {  // two multiply-shift divisions per block
      r = decode_row<MODE>(p, m0 + b * kBlockM + row_in_block);
      decoded_b = b;
    }
    // the residual is in flight together with the TMEM load
    const uint4 x = (KIND == kEpiResidual || KIND == kEpiGeneric) ? residual_load(p, r, ntile, j) : make_uint4(0, 0, 0, 0);
    tmem_ld_wait();
    // reset the drained columns to the bias for the next tile's MMAs, which all accumulate
    tmem_fill16(c, bias4_s + j * 4);
    if (KIND == kEpiGeneric) {
      if (p.pre_shift) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = pre_reduce(v[i], p.pre_shift);
      }
      if (r.valid) store_piece(p, r, ntile, j, v, x, lut_s, scale, rscale, linear);
    } else if (KIND == kEpiLinearNCHW) {
      // a detect head: linear, int8 NCHW into the egress; a warp's 32 rows are 32 pixels, so each
      // byte store covers up to 32 consecutive bytes of one channel plane
      const uint4 o = epilogue16_linear(v, scale);
      if (r.valid) {
        int8_t* e = p.egress + (long long)r.img * p.egress_img + r.oy * p.Wo + r.ox;
        const long long plane = (long long)p.Ho * p.Wo;
        const int8_t* ob = reinterpret_cast<const int8_t*>(&o);
        const int c0 = ntile * p.n_tile + j * 16;
        if (c0 + 16 <= p.egress_ch) {
#pragma unroll
          for (int i = 0; i < 16; ++i) e[(c0 + i) * plane] = ob[i];
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (c0 + i < p.egress_ch) e[(c0 + i) * plane] = ob[i];
        }
      }
    } else if (KIND == kEpiTableS2D) {
      // table layer whose consumer is a stride-2 conv: its space-to-depth copy, and the plain
      // output unless nothing else reads it
      const uint4 o = epilogue16<false>(v, lut_s, scale, p, rscale, x);
      if (r.valid) {
        const int oc = ntile * nj + j;
        if (p.out2_kind != IXB_OUT2_S2D_ONLY)
          *reinterpret_cast<uint4*>(const_cast<int8_t*>(p.out.base) + (long long)oc * p.out.plane +
                                    (long long)r.opix * 16) = o;
        const int ph = (r.oy & 1) * 2 + (r.ox & 1);
        *reinterpret_cast<uint4*>(const_cast<int8_t*>(p.out2.base) + (long long)(ph * (p.cout >> 4) + oc) * p.out2.plane +
                                  ((long long)r.img * p.out2.P + (long long)((r.oy >> 1) + 1) * (p.out2.W + 2) +
                                   (r.ox >> 1) + 1) * 16) = o;
      }
    } else {
      // every lane computes (halo rows too: their residual reads as zero), only valid rows store,
      // so the arithmetic is not a divergent branch
      uint4 o;
      if (KIND == kEpiLinear)
        o = epilogue16_linear(v, scale);
      else
        o = epilogue16<KIND == kEpiResidual>(v, lut_s, scale, p, rscale, x);
      if (r.valid)
        *reinterpret_cast<uint4*>(const_cast<int8_t*>(p.out.base) + (long long)(ntile * nj + j) * p.out.plane +
                                  (long long)r.opix * 16) = o;
    }
    if (++j == nj) {
      j = 0;
      ++b;
    }
  }
  tmem_st_wait();  // the biases are in TMEM before the accumulator is handed back
}

// The epilogue warps' loop over the CTA's tiles: wait for an accumulator, drain it, hand it back.
template <int MODE, int EW, int KIND>
__device__ __forceinline__ void epilogue_role(const ConvParams& p, uint64_t* acc_full, uint64_t* acc_empty,
                                              uint32_t tmem, int ntile, int warp, int lane, const uint8_t* lut_s,
                                              const int4* bias4_s, bool linear) {
  int acc = 0;
  uint32_t aph = 0;
  long long ew = 0, ek = 0;
  int tiles = 0;
  for (int t = blockIdx.x; t < p.m_tiles; t += gridDim.x) {
    const long long c0 = clock64();
    mbar_wait(&acc_full[acc], aph);
    const long long c1 = clock64();
    ew += c1 - c0;
    tc_fence_after();
    conv_epilogue_tile<MODE, EW, KIND>(p, tmem + acc * p.acc_cols, t * p.tile_rows, ntile, warp, lane, lut_s,
                                       bias4_s, tiles, linear);
    tc_fence_before();
    mbar_arrive(&acc_empty[acc]);
    ek += clock64() - c1;
    ++tiles;
    if (++acc == p.nacc) {
      acc = 0;
      aph ^= 1;
    }
  }
  if (threadIdx.x == 0) {
    write_stats(p, kStatEpiWait, ew);
    write_stats(p, kStatEpiWork, ek);
    write_stats(p, kStatTiles, tiles);
  }
}

template <int MODE, int EW>
__global__ void __launch_bounds__(conv_threads(MODE, EW), 1) conv_kernel(const __grid_constant__ ConvParams p) {
  constexpr int EPI = EW, PW0 = EPI, MW0 = mma_warp0(MODE, EW);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + p.nacc;
  uint64_t* bres_bar = acc_empty + p.nacc;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres_bar + 1);
  __shared__ uint8_t lut_tab[256];  // static: the epilogue indexes it from a constant address
  const uint8_t* lut_s = lut_tab + 128;
  int* bias_s = reinterpret_cast<int*>(smem + p.bias_off);
  const int4* bias4_s = reinterpret_cast<const int4*>(smem + p.bias_off);
  const int ntile = blockIdx.y;
  const int KB = p.kblocks;
  const long long t_start = clock64();
  grid_dep_launch();
  if (tid == 0) trace_mark(p.trace, 0);

  if (warp == 0) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  if (tid == MW0 * 32) {
    const uint32_t fcount = (MODE == IXB_MODE_GATHER) ? (uint32_t)kGatherThreads + (p.b_resident ? 0u : 1u) : 1u;
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], fcount);
      mbar_init(&empty[s], p.issuers);  // every issuer commits every stage
    }
    for (int b = 0; b < p.nacc; ++b) {
      mbar_init(&acc_full[b], p.issuers);
      mbar_init(&acc_empty[b], EPI * 32);
    }
    mbar_init(bres_bar, 1);
    fence_mbar_init();
  }
  if (MODE == IXB_MODE_IM2COL || MODE == IXB_MODE_STEM) {
    if (tid == PW0 * 32) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tmap) : "memory");
  }
  for (int i = tid; i < 256; i += conv_threads(MODE, EW)) lut_tab[i] = (uint8_t)p.lut[i];
  // a linear layer's table is the identity (entry i holds i - 128): its epilogue skips the lookups.
  // Thread i < 256 wrote entry i itself, so each reads its own write.
  const bool linear = __syncthreads_and(tid >= 256 || lut_tab[tid] == (uint8_t)(tid - 128)) != 0;
  for (int i = tid; i < p.n_tile; i += conv_threads(MODE, EW)) bias_s[i] = p.bias[ntile * p.n_tile + i];
  if (MODE == IXB_MODE_WINDOW) {
    const int8_t** ctab = reinterpret_cast<const int8_t**>(smem + p.ctab_off);
    for (int gc = tid; gc < p.cin_chunks; gc += conv_threads(MODE, EW)) {
      const SegDev& s = p.seg[seg_of_chunk(p, gc)];
      ctab[gc] = s.base + (long long)(gc - s.chunk_begin) * s.plane;
    }
  }
  if (MODE == IXB_MODE_GATHER) {
    GatherChunk* gtab = reinterpret_cast<GatherChunk*>(smem + p.ctab_off);
    for (int gc = tid; gc < p.cin_chunks; gc += conv_threads(MODE, EW)) {
      const SegDev& s = p.seg[seg_of_chunk(p, gc)];  // the host checks that the segments tile the chunks
      gtab[gc] = GatherChunk{s.base + (long long)(gc - s.chunk_begin) * s.plane, s.P, s.W + 2, s.up2, 0};
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < EPI) {
    // every accumulator starts at the bias: every MMA accumulates (see issue_mma)
    const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
    for (int c = (warp >> 2) * 16; c < p.nacc * p.acc_cols; c += (EPI / 4) * 16)
      tmem_fill16(tmem + lanes + (uint32_t)c, bias4_s + ((c % p.n_tile) >> 4) * 4);
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  if (warp >= PW0 && warp < MW0) {
    // ------------------------------------------------------------ producers
    const int ptid = tid - PW0 * 32;
    if (p.b_resident && ptid == 0) {
      const int total = p.kb[KB - 1].b_off + p.kb[KB - 1].b_bytes;
      mbar_arrive_expect_tx(bres_bar, (uint32_t)total);
      for (int kb = 0; kb < KB; ++kb)
        bulk_g2s(smem + p.kb[kb].b_off, p.wpack + ntile * p.w_ntile_stride + p.kb[kb].b_off, p.kb[kb].b_bytes, bres_bar);
    }
    grid_dep_wait();  // activations of the previous layer from here on
    if (ptid == 0) trace_mark(p.trace, 1);
    if (MODE == IXB_MODE_GATHER) {
      produce_gather(p, smem, full, empty, ntile, ptid);
    } else if (ptid == 0) {
      produce_single<MODE>(p, smem, full, empty, ntile);
    }
  } else if (warp >= MW0) {
    // ------------------------------------------------------------ MMA issuers
    const int who = __shfl_sync(0xffffffffu, warp - MW0, 0);  // warp-uniform for the compiler
    if (who < p.issuers)
      issue_mma<MODE>(p, smem, full, empty, acc_full, acc_empty, bres_bar, tmem, who);
  } else {
    // ------------------------------------------------------------ epilogue
    grid_dep_wait();  // residual reads and output writes follow the previous layer
    if (p.pre_shift)  // SRS shifts above 16: the generic drain, which pre-reduces exactly
      epilogue_role<MODE, EW, kEpiGeneric>(p, acc_full, acc_empty, tmem, ntile, warp, lane, lut_s, bias4_s, linear);
    else if (p.out_nchw && !p.has_res && linear)
      epilogue_role<MODE, EW, kEpiLinearNCHW>(p, acc_full, acc_empty, tmem, ntile, warp, lane, lut_s, bias4_s, linear);
    else if (!p.out_nchw && !p.has_res && !linear && p.out2_kind >= IXB_OUT2_S2D)
      epilogue_role<MODE, EW, kEpiTableS2D>(p, acc_full, acc_empty, tmem, ntile, warp, lane, lut_s, bias4_s, linear);
    else if (p.out_nchw || p.out2_kind)
      epilogue_role<MODE, EW, kEpiGeneric>(p, acc_full, acc_empty, tmem, ntile, warp, lane, lut_s, bias4_s, linear);
    else if (p.has_res)
      epilogue_role<MODE, EW, kEpiResidual>(p, acc_full, acc_empty, tmem, ntile, warp, lane, lut_s, bias4_s, linear);
    else if (linear)
      epilogue_role<MODE, EW, kEpiLinear>(p, acc_full, acc_empty, tmem, ntile, warp, lane, lut_s, bias4_s, linear);
    else
      epilogue_role<MODE, EW, kEpiTable>(p, acc_full, acc_empty, tmem, ntile, warp, lane, lut_s, bias4_s, linear);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, p.tmem_cols);
  if (tid == 0) write_stats(p, kStatTotal, clock64() - t_start);
  if (tid == 0) trace_mark(p.trace, 2);
}

}  // namespace ixb
