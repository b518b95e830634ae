// int8 GEMM on the 5th-generation tensor cores (tcgen05, kind::i8) with the pow2 SRS epilogue,
// and its raw int32 form.
//
//   out[m][n] = clamp(rne((sum_k a[m][k] * b[n][k] + bias[n]) >> shift), -128, 127)   (SRS)
//   out[m][n] = sum_k a[m][k] * b[n][k]                                               (I32)
//
// Both are exact for K <= 65536, any int32 bias and shift <= 23: the product cannot overflow
// int32, and a bias sum that would is saturated, which clamps to the same int8.
//
// a is int8 [M][K] row-major; b is int8 [N][K], i.e. B of C = A.B given K-major (the layout
// int8 tensor-core GEMMs take). The rounding is round-half-to-even and the clamp saturates,
// the SRS rule of the reference's engine (engine_emulator.py:149-162, engine.cc:186-191);
// the int32 product is the exact integer GEMM of kernels/int8_matmul_sweep.
//
// Persistent and warp-specialised: one thread issues TMA tile loads (A: MT boxes of 128 rows x
// 128 bytes of K, B: one box of BN rows x 128 bytes, both 128-byte swizzled), one thread issues
// tcgen05.mma (M = 128 per block, N = BN, K = 32 per instruction, four per stage), and EPI warps
// drain the two TMEM accumulators (MT blocks x BN columns each) through the integer epilogue, so
// the epilogue of tile i overlaps the MMAs of tile i + 1. TMA zero-fills rows past M or N and K
// past its end, so ragged shapes need no padding in memory.
#pragma once
#include <cstdint>
#include <cuda.h>
#include "ixb_ptx.cuh"
#include "ixb_w4a8.cuh"

namespace ixb {

constexpr int kGemmBK = 128;                 // K bytes per stage: one 128-byte swizzle row
constexpr int kGemmABlock = 128 * kGemmBK;   // one 128-row A box
constexpr int kGemmMaxStages = 8;
enum : int { GEMM_OUT_SRS = 0, GEMM_OUT_I32 = 1 };

struct GemmParams {
  alignas(64) CUtensorMap ta;  // A [M][K], box {128 B, 128 rows}, SWIZZLE_128B
  alignas(64) CUtensorMap tb;  // B [N][K], box {128 B, BN rows}, SWIZZLE_128B; W4A8: the packed
                               // weights [N][K/2], box {64 B, BN rows}, no swizzle
  int M, N, K;
  int bn, mt, m_tiles, n_tiles, kblocks, stages;
  int stage_bytes, stage_tx, bar_off;
  int raw_off;               // W4A8: offset of the packed int4 B tile inside a stage
  int eg_off;                // W4A8: the tile's group exponents [BN][K/128] in shared memory, or -1
                             // (read from global memory) when they would not fit
  int acc_cols, tmem_cols, nacc;  // TMEM accumulators of acc_cols columns (1 or 2)
  uint32_t idesc;
  int out_kind;
  const int32_t* bias;
  int shift;
  int8_t* out8;
  int32_t* out32;
  // W4A8 (B from the packed int4 weight image, unpacked by the B warps)
  const uint8_t* wq;         // [N][K/2]
  const uint8_t* eg;         // [N][K/128]
  const int32_t* shift_vec;  // per output column, or null for `shift`
};

// K-major operand in the 128-byte swizzle layout TMA writes: rows of 128 bytes, 8-row atoms of
// 1024 bytes (SBO), 16-byte chunks XOR-permuted by the row within the atom. Successive 32-byte
// K steps advance the start address inside the atom.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;                // LBO: unused by swizzled K-major layouts
  d |= (uint64_t)(1024 >> 4) << 32;      // SBO: next 8-row atom
  d |= (uint64_t)1 << 46;                // descriptor version for sm_100
  d |= (uint64_t)2 << 61;                // layout: 128-byte swizzle
  return d;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

enum : int { GEMM_B_TMA = 0, GEMM_B_W4 = 1 };
constexpr int kW4Warps = 8;  // warps unpacking int4 weights into the B stage (GEMM_B_W4): two per SM sub-partition
constexpr int gemm_threads(int epi, int bsrc) { return 32 * (epi + 2 + (bsrc == GEMM_B_W4 ? kW4Warps : 0)); }

// B warps of the W4A8 GEMM: per stage the TMA has brought the packed int4 tile (BN rows x 64
// bytes = 128 values of K, one group) into shared memory with the A boxes; the warps turn it
// into the int8 B operand, 16 values (8 packed bytes) per item into one 16-byte chunk of the
// 128-byte swizzled row (chunk c at c ^ (row % 8)), scaled by the group's 2^-e. Reading the packed
// tile from shared memory keeps global-memory latency out of the unpack loop.
__device__ __forceinline__ void produce_w4(const GemmParams& p, uint8_t* smem, uint64_t* full, uint64_t* bfull,
                                           int ut) {
  constexpr int UT = kW4Warps * 32;
  const int S = p.stages, G = p.K / 128;
  const int tiles = p.m_tiles * p.n_tiles;
  const int items = 8 * p.bn;
  uint8_t* eg_s = p.eg_off >= 0 ? smem + p.eg_off : nullptr;
  int s = 0;
  uint32_t ph = 0;
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int ntile = t % p.n_tiles;
    const int n0 = ntile * p.bn;
    if (eg_s) {
      // the tile's group exponents, one contiguous run of [N][K/128], once per tile (the 128 B-warp
      // threads meet on named barrier 2 around the refill; no thread leaves this loop early)
      asm volatile("bar.sync 2, %0;" ::"n"(UT) : "memory");
      const long long e0 = (long long)n0 * G, e1 = (long long)min(n0 + p.bn, p.N) * G;
      for (long long i = e0 + ut; i < e1; i += UT) eg_s[i - e0] = __ldg(p.eg + i);
      asm volatile("bar.sync 2, %0;" ::"n"(UT) : "memory");
    }
    for (int kb = 0; kb < p.kblocks; ++kb) {
      const bool ok = mbar_wait(&full[s], ph);  // a timeout raised the device flag; the loop runs on
      uint8_t* st = smem + s * p.stage_bytes;
      uint8_t* bst = st + p.mt * kGemmABlock;
      const uint8_t* raw = st + p.raw_off;
      for (int i = ut; ok && i < items; i += UT) {
        const int r = i >> 3, c = i & 7;
        const int n = n0 + r;
        const uint2 w = *reinterpret_cast<const uint2*>(raw + r * 64 + c * 8);  // zero past N (TMA fill)
        const uint32_t e = n >= p.N ? 0u : (eg_s ? (uint32_t)eg_s[r * G + kb] : (uint32_t)__ldg(p.eg + (long long)n * G + kb));
        uint4 o = make_uint4(w4_lo16(w.x), w4_hi16(w.x), w4_lo16(w.y), w4_hi16(w.y));
        if (e) {
          const uint32_t keep = (0xFFu >> e) * 0x01010101u;
          const uint32_t fill = ((0xFFu << (8 - e)) & 0xFFu);
          o.x = sra8_lanes(o.x, e, keep, fill);
          o.y = sra8_lanes(o.y, e, keep, fill);
          o.z = sra8_lanes(o.z, e, keep, fill);
          o.w = sra8_lanes(o.w, e, keep, fill);
        }
        *reinterpret_cast<uint4*>(bst + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)) = o;
      }
      fence_proxy_async_smem();  // generic-proxy stores -> tensor-core reads
      mbar_arrive(&bfull[s]);
      if (++s == S) {
        s = 0;
        ph ^= 1;
      }
    }
  }
}

template <int EPI, int BSRC>
__global__ void __launch_bounds__(gemm_threads(EPI, BSRC), 1) gemm_kernel(const __grid_constant__ GemmParams p) {
  constexpr int PW = EPI, MW = EPI + 1, UW0 = EPI + 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.bar_off);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done = acc_empty + 2;
  uint64_t* bfull = done + 1;  // W4A8: the stage's B operand is unpacked
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bfull + kGemmMaxStages);
  const int tiles = p.m_tiles * p.n_tiles;

  if (warp == MW) {
    tmem_alloc(tmem_slot, p.tmem_cols);
    tmem_relinquish();
  }
  if (tid == PW * 32) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&bfull[s], kW4Warps * 32);
    }
    for (int b = 0; b < p.nacc; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI * 32);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.ta) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tb) : "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == PW) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int mtile = t / p.n_tiles, ntile = t - mtile * p.n_tiles;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * p.stage_bytes;
          mbar_arrive_expect_tx(&full[s], (uint32_t)p.stage_tx);
          for (int b = 0; b < p.mt; ++b)
            tma_load_2d(st + b * kGemmABlock, &p.ta, kb * kGemmBK, (mtile * p.mt + b) * 128, &full[s]);
          if (BSRC == GEMM_B_TMA) tma_load_2d(st + p.mt * kGemmABlock, &p.tb, kb * kGemmBK, ntile * p.bn, &full[s]);
          else tma_load_2d(st + p.raw_off, &p.tb, kb * (kGemmBK / 2), ntile * p.bn, &full[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (BSRC == GEMM_B_W4 && warp >= UW0) {
    // ------------------------------------------------------------ int4 -> int8 B producers
    produce_w4(p, smem, full, bfull, tid - UW0 * 32);
  } else if (warp == MW) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      bool issued = false;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        if (!mbar_wait(&acc_empty[acc], aph ^ 1)) break;
        tc_fence_after();
        const uint32_t d0 = tmem + acc * p.acc_cols;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&full[s], ph) || (BSRC == GEMM_B_W4 && !mbar_wait(&bfull[s], ph))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + s * p.stage_bytes);
          const int ksteps = min(kGemmBK / 32, (p.K - kb * kGemmBK + 31) / 32);
          for (int j = 0; j < ksteps; ++j) {
            const uint64_t bd = umma_desc_sw128(st + p.mt * kGemmABlock + j * 32);
            for (int b = 0; b < p.mt; ++b)
              umma_s8(d0 + b * p.bn, umma_desc_sw128(st + b * kGemmABlock + j * 32), bd, p.idesc,
                      (kb | j) != 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(&empty[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        if (++acc == p.nacc) {
          acc = 0;
          aph ^= 1;
        }
      }
      if (issued) {
        umma_commit(done);  // every MMA this CTA issued has finished before TMEM is released
        mbar_wait(done, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int NG = EPI / 4;
    const int q = warp & 3, g = warp >> 2;
    const int nch = p.bn / 16;
    const int s = p.shift, hs = s > 0 ? (1 << (s - 1)) - 1 : 0, lsb = s > 0 ? 1 : 0;
    // shifts up to 16 round through the float unit (exact: see the conv epilogue's srs_s8)
    const bool fsrs = s <= 16;
    const float fscale = __int_as_float((127 - (fsrs ? s : 0)) << 23);
    int acc = 0;
    uint32_t aph = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      if (!mbar_wait(&acc_full[acc], aph)) break;
      tc_fence_after();
      const int mtile = t / p.n_tiles, ntile = t - mtile * p.n_tiles;
      const uint32_t base = tmem + acc * p.acc_cols + ((uint32_t)(q * 32) << 16);
      for (int k = g; k < p.mt * nch; k += NG) {
        const int b = k / nch, c = k - b * nch;
        uint32_t v[16];
        tmem_ld16(base + b * p.bn + c * 16, v);
        tmem_ld_wait();
        const int row = (mtile * p.mt + b) * 128 + q * 32 + lane;
        const int col = ntile * p.bn + c * 16;
        if (row >= p.M || col >= p.N) continue;
        if (p.out_kind == GEMM_OUT_I32) {
          uint4* o = reinterpret_cast<uint4*>(p.out32 + (long long)row * p.N + col);
#pragma unroll
          for (int i = 0; i < 4; ++i) o[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else if (p.shift_vec) {
          // W4A8: no bias, one shift per output column
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t packed = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int r = clamp_i8(rne_shift((int)v[4 * i + e], __ldg(p.shift_vec + col + 4 * i + e)));
              packed |= (uint32_t)(r & 0xFF) << (8 * e);
            }
            w[i] = packed;
          }
          *reinterpret_cast<uint4*>(p.out8 + (long long)row * p.N + col) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
          const int4* b4 = reinterpret_cast<const int4*>(p.bias + col);
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int4 bb = __ldg(b4 + i);
            const int bv[4] = {bb.x, bb.y, bb.z, bb.w};
            uint32_t packed = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // saturating adds: a sum past int32 saturates, which for shift <= 23 still clamps
              // to the same int8 as the exact value
              const int a = add_sat((int)v[4 * i + e], bv[e]);
              int r;
              if (fsrs) {
                asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(__int2float_rn(a) * fscale));
                r = (int)(int8_t)r;
              } else {
                r = clamp_i8(add_sat(a, hs + ((a >> s) & lsb)) >> s);
              }
              packed |= (uint32_t)(r & 0xFF) << (8 * e);
            }
            w[i] = packed;
          }
          *reinterpret_cast<uint4*>(p.out8 + (long long)row * p.N + col) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == p.nacc) {
        acc = 0;
        aph ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == MW) tmem_dealloc(tmem, p.tmem_cols);
}

}  // namespace ixb
