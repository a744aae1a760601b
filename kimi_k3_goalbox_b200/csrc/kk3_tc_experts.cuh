// Routed-expert engine on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Not on the decode-step path: the step runs the warp-level mma.sync engine (run_experts, kk3_gemv.cuh),
// which streams the experts as fast as this one at decode batch sizes (measured per-operation costs below).
// kk3_tc_check.cu runs both engines on the same routed batch and checks that their results agree.
//
// The MXFP4 expert weights (e2m1 codes [E, rows, K/2] + E8M0 scales [E, rows, K/32], kimi.py:116-119,
// quantization.py:38-52) are multiplied by tcgen05.mma kind::mxf8f6f4.block_scale: the tensor core decodes
// the 4-bit codes and applies both operands' per-32 E8M0 scales itself, so no thread converts a weight.
//
//  - A (weights): one 256-row x 128-k tile per matrix and k-step, ONE TMA box with the 16U4_ALIGN16B
//    element type (16 codes in every 16-byte smem chunk) into the 128-byte-swizzled K-major layout; its two
//    128-row halves are two M = 128 MMAs. Rows past the matrix (a last partial tile) are zero-filled by TMA.
//  - B (activations): the bf16-valued activations as two E4M3 terms with their own per-32 E8M0 scales,
//    x = 2^(s1-127) q1 + 2^(s2-127) q2. q1 carries the top four significant bits and q2 the remaining four,
//    so every element within 2^13 of its block's maximum is represented exactly (an activation has eight
//    significant bits). One row per (expert, token) pair. The terms live in global "images" laid out as
//    the smem operand: per 128-k step and 8-pair atom, the 8 rows of term 0 then the 8 rows of term 1
//    (128-byte rows, 16-byte chunks XOR-swizzled by the row), so that the pair window of a chunk (one or two
//    atoms) is one contiguous 1-D bulk copy and both terms go through ONE MMA as separate columns
//    (N = 2 x window); the epilogue adds the two columns of each pair.
//  - Scale factors: weight scales are gathered by the producer warp into the 32x128b layout that
//    tcgen05.cp ... warpx4 replicates into all four TMEM lane quarters (row m0 + 32 m1 at smem byte
//    16 m0 + 4 m1 + kb); activation scales come from the images in the same layout.
//  - D: FP32 accumulators in TMEM (128 lanes = rows of a tile half, one column per activation row and
//    term), double-buffered so that the epilogue of one tile overlaps the MMAs of the next.
//
// Work split: stream-K over units (expert chunk, 256-row tile, 128-k step), a contiguous range per CTA. A
// tile whose units span several CTAs is finished by the last contributor to arrive, which sums every
// contributor's partial in CTA order (deterministic). Roles inside a CTA: warps 0 and 2 produce alternate
// units (scale gather, then TMA / bulk issue by lane 0), lane 0 of warp 1 issues tcgen05.cp / tcgen05.mma, warps 4-11 read the
// accumulators (warp 4 + 4h + q owns TMEM lanes 32q..32q+31 of half h) and run the epilogue. Each TMA or
// bulk copy costs a fixed issue time, so the units are as large as shared memory allows (one 256-row box
// per matrix). Every wait is bounded.
//
// Measured limits on B200 (TP8-rank geometry, b8): a TMA / bulk operation occupies an SM's copy engine for
// ~0.3 us whatever its size (4-32 KB), a 16U4 box carries at most 16 KB of codes, and an M = 128, N = 16,
// K = 32 block-scaled MMA issues every ~45 ns; a 32 KB unit of gate/up codes therefore costs ~1 us.
// Keeping one unit's scale writes and its copy issue in the same warp matters: a variant that gathered the
// scales in a separate warp produced wrong down-projection results (deterministically, with identical
// shared-memory operands), so the two producer warps here each own whole units.
#pragma once
#include <cuda.h>
#include "kk3_phases.cuh"
#include "kk3_tcgen05.cuh"

namespace kk3 {

constexpr int kTcTerms = 2;          // E4M3 terms per activation
constexpr int kTcMaxStages = 8;
constexpr int kTcRows = 256;         // rows of a weight tile: one TMA box, two M = 128 MMAs per k-block
constexpr int kTcTmemCols = 512;     // accumulators + scale factors (one CTA per SM)
constexpr int kTcDCols = 256;        // accumulators: 2 buffers x MT x 2 halves x N (N <= 32)
constexpr int kTcChunkCache = 64;    // chunk descriptors cached in shared memory per CTA

// Per-phase descriptor of the tensor-core expert engine.
struct TcPhase {
  const CUtensorMap* map[2];     // codes of matrix 0/1 (gate, up) or (down, -): 3-D {K, rows, E} of 4-bit codes
  const uint8_t* scales[2];      // E8M0 [E, rows, K/32]
  int rows, K, tiles, ksteps;    // tiles = ceil(rows / 256), ksteps = K / 128
  long long expert_scales;       // rows * K / 32
  const uint8_t* bimg;           // activation image [ksteps][atoms][terms][8][128] (E4M3, swizzled rows)
  const uint8_t* bsfb;           // its scales [ksteps][atoms][terms][8][16] (bytes 0..3 = the 4 k-blocks)
  int atoms;                     // 8-pair atoms of the images (pairs rounded up to 8, / 8)
  float* part;                   // [grid][2][MT][8][256] stream-K partial tiles
  int* cnt;                      // [chunks * tiles] arrival counters (left at zero)
  uint8_t* oimg;                 // MT == 2: output image of the activations (the down projection's B)
  uint8_t* osfb;                 //   and its scales (same layouts, ksteps = rows / 128)
  __half* act_dbg;               // MT == 2: optional FP16 copy of the activations [pairs, rows]
};

// ---- PTX wrappers (the shared ones are in kk3_tcgen05.cuh) -------------------------------------------

KK3_DEV void tma_load_3d(unsigned dst, const CUtensorMap* map, unsigned bar, int x, int y, int z,
                         unsigned long long pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;"
      ::"r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z), "l"(pol) : "memory");
}
KK3_DEV void bulk_load(unsigned dst, const void* src, unsigned bytes, unsigned bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
// 32 rows x 16 bytes of shared memory -> TMEM lanes 32w + row (every w), 4 columns
KK3_DEV void tmem_cp_32x128b_x4(unsigned taddr, unsigned long long sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
KK3_DEV void umma_mxf8f6f4(unsigned d, unsigned long long adesc, unsigned long long bdesc, unsigned idesc,
                           unsigned sfa, unsigned sfb, unsigned accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n}"
      ::"r"(d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb) : "memory");
}
// no swizzle, 16-byte rows, 8-row core matrices 128 bytes apart (the 32x128b scale-factor source)
KK3_DEV unsigned long long sdesc_rows16(unsigned addr) {
  return (unsigned long long)((addr & 0x3ffffu) >> 4) | (1ull << 16) | ((unsigned long long)(128 >> 4) << 32) |
         (1ull << 46);
}
// Instruction descriptor: kind::mxf8f6f4, A = E2M1, B = E4M3, D = F32, both K-major, E8M0 scales, M = 128.
// Scale-factor ids select the byte (k-block) inside each 32-bit TMEM scale column.
KK3_DEV unsigned idesc_mxf4_e4m3(int n, unsigned sf_id) {
  return (sf_id << 4) | (5u << 7) | (0u << 10) | ((unsigned)(n >> 3) << 17) | (1u << 23) | ((128u >> 4) << 24) |
         (sf_id << 29);
}

// ---- activation quantisation ---------------------------------------------------------------------------

KK3_DEV unsigned f32_to_e4m3(float x) {
  unsigned short r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(x));
  return r & 0xffu;
}
KK3_DEV float e4m3_to_f32(unsigned q) {
  unsigned r;
  const unsigned short in = (unsigned short)q;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(in));
  return __half2float(__ushort_as_half((unsigned short)(r & 0xffffu)));
}
// block exponent: the block maximum lands in [128, 256) after scaling by 2^-e (e in [-126, 126], so that
// 2^-e is a normal float and the E8M0 byte e + 127 is in [1, 253])
KK3_DEV int tc_block_exp(float amax) {
  if (!(amax > 0.0f)) return 0;
  int e = (int)((__float_as_uint(amax) >> 23) & 0xffu) - 127 - 7;
  return e < -126 ? -126 : (e > 126 ? 126 : e);
}
// One value per lane, the warp's 32 lanes forming one 32-wide block: two E4M3 terms and their E8M0 bytes.
KK3_DEV void tc_quant2(float v, unsigned& q1, unsigned& q2, unsigned& s1, unsigned& s2) {
  const int e1 = tc_block_exp(warp_max(fabsf(v)));
  q1 = f32_to_e4m3(v * __uint_as_float((unsigned)(127 - e1) << 23));
  const float r = v - e4m3_to_f32(q1) * __uint_as_float((unsigned)(127 + e1) << 23);
  const int e2 = tc_block_exp(warp_max(fabsf(r)));
  q2 = f32_to_e4m3(r * __uint_as_float((unsigned)(127 - e2) << 23));
  s1 = (unsigned)(e1 + 127);
  s2 = (unsigned)(e2 + 127);
}
// image offsets of pair row p, term t, k-step ks, k in [0, 128) (block k >> 5)
KK3_DEV size_t tc_img_off(int atoms, int ks, int p, int t, int k) {
  const unsigned r = (unsigned)p & 7u;
  return ((((size_t)ks * atoms + (p >> 3)) * kTcTerms + t) << 10) + r * 128u +
         (((((unsigned)k >> 4) ^ r)) << 4) + ((unsigned)k & 15u);
}
KK3_DEV size_t tc_sfb_off(int atoms, int ks, int p, int t, int k) {
  return ((((size_t)ks * atoms + (p >> 3)) * kTcTerms + t) << 7) + ((unsigned)p & 7u) * 16u + ((unsigned)k >> 5);
}
KK3_DEV void tc_store_terms(uint8_t* img, uint8_t* sfb, int atoms, int ks, int p, int k, float v) {
  unsigned q[2], s[2];
  tc_quant2(v, q[0], q[1], s[0], s[1]);
#pragma unroll
  for (int t = 0; t < kTcTerms; ++t) {
    img[tc_img_off(atoms, ks, p, t, k)] = (uint8_t)q[t];
    if ((threadIdx.x & 31) == 0) sfb[tc_sfb_off(atoms, ks, p, t, k)] = (uint8_t)s[t];
  }
}

// Activation image of the gate/up projection: pair p's row is the FP16 latent row of its token. Every warp
// of the grid quantises 32-wide blocks (lane = element); rows of the last atom beyond the pairs are zero.
KK3_DEV void tc_quant_pairs(const StepArgs& a, const __half* x, int K, int npairs, int atoms, uint8_t* img, uint8_t* sfb) {
  const int lane = threadIdx.x & 31;
  const int nblk = K >> 5;
  const long long items = (long long)atoms * 8 * nblk;
  const long long gw = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long it = gw; it < items; it += nw) {
    const int p = (int)(it / nblk), blk = (int)(it - (long long)p * nblk);
    const int k = blk * 32 + lane;
    float v = 0.0f;
    if (p < npairs) {
      int b = __ldcg(a.s.pair_row + p);
      b = b < 0 ? 0 : (b >= a.g.B ? a.g.B - 1 : b);
      v = __half2float(x[(size_t)b * K + k]);
    }
    tc_store_terms(img, sfb, atoms, k >> 7, p, k & 127, v);
  }
}

// ---- the engine --------------------------------------------------------------------------------------

template <int MT>
__host__ __device__ constexpr int tc_stage_bytes() {
  // A[MT] 32 KB each | B: 2 atoms x 2 terms x 1 KB | SFA[MT][2 halves] 512 B | SFB 512 B
  return (MT * 32768 + 4096 + (2 * MT + 1) * 512 + 1023) & ~1023;
}

// unit iterator: (chunk, tile, k-step) in unit order, no divisions after the start
struct TcIter {
  int chunk, tile, ks;
};

template <int MT>
KK3_FN void run_experts_tc(const StepArgs& a, const TcPhase& ph, int smem_bytes) {
  extern __shared__ __align__(1024) unsigned char kk3_dyn_smem[];
  constexpr int kTcBars = 2 * kTcMaxStages + 5;   // full[S], empty[S], acc full[2], acc empty[2], drain
  constexpr int kEpiWarps = 8, kEpiThreads = kEpiWarps * 32;
  __shared__ __align__(8) unsigned long long tc_bar[kTcBars];
  __shared__ unsigned tc_tmem;
  __shared__ int tc_last;
  __shared__ int tc_run;   // one decision for the whole CTA: every role runs, or none
  __shared__ int s_cexp[kTcChunkCache], s_cfp[kTcChunkCache], s_cnp[kTcChunkCache];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int npk = a.g.B * a.g.K;
  int nchunks = __ldcg(a.s.chunk_info);
  nchunks = nchunks < 0 ? 0 : (nchunks > npk ? npk : nchunks);
  const int tiles = ph.tiles, ksteps = ph.ksteps, per_chunk = tiles * ksteps;
  const int U = nchunks * per_chunk;
  if (U == 0) return;                               // the same for every thread of the grid
  const int G = (int)gridDim.x < U ? (int)gridDim.x : U;
  if ((int)blockIdx.x >= G) return;                 // the whole CTA
  const int ubeg = (int)((long long)U * blockIdx.x / G), uend = (int)((long long)U * (blockIdx.x + 1) / G);
  const int nunits = uend - ubeg;
  TcIter it0;
  it0.chunk = ubeg / per_chunk;
  {
    const int rem = ubeg - it0.chunk * per_chunk;
    it0.tile = rem / ksteps;
    it0.ks = rem - it0.tile * ksteps;
  }
  const int c_lo = it0.chunk;
  auto step = [&](TcIter& t) {
    if (++t.ks == ksteps) {
      t.ks = 0;
      if (++t.tile == tiles) {
        t.tile = 0;
        ++t.chunk;
      }
    }
  };

  // chunk descriptors of this CTA's range (clamped so that a routing fault cannot address outside buffers)
  auto load_chunk = [&](int chunk, int& e, int& fp, int& np) {
    e = __ldcg(a.s.chunk_info + 1 + chunk * 3);
    fp = __ldcg(a.s.chunk_info + 2 + chunk * 3);
    np = __ldcg(a.s.chunk_info + 3 + chunk * 3);
    e = e < 0 ? 0 : (e >= a.g.E ? a.g.E - 1 : e);
    fp = fp < 0 ? 0 : (fp >= npk ? npk - 1 : fp);
    np = np < 0 ? 0 : (np > 8 ? 8 : np);
    np = fp + np > npk ? npk - fp : np;
  };
  for (int i = threadIdx.x; i < kTcChunkCache; i += blockDim.x) {
    int e = 0, fp = 0, np = 0;
    if (c_lo + i < nchunks) load_chunk(c_lo + i, e, fp, np);
    s_cexp[i] = e;
    s_cfp[i] = fp;
    s_cnp[i] = np;
  }
  auto chunk_info = [&](int chunk, int& e, int& fp, int& np) {
    const int i = chunk - c_lo;
    if (i < kTcChunkCache) {
      e = s_cexp[i];
      fp = s_cfp[i];
      np = s_cnp[i];
    } else {
      load_chunk(chunk, e, fp, np);
    }
  };

  const unsigned dyn = smem_u32(kk3_dyn_smem);
  const unsigned base = (dyn + 1023u) & ~1023u;
  const int stage_bytes = tc_stage_bytes<MT>();
  int S = (smem_bytes - (int)(base - dyn)) / stage_bytes;
  S = S > kTcMaxStages ? kTcMaxStages : S;
  constexpr unsigned off_b = MT * 32768, off_sfa = off_b + 4096, off_sfb = off_sfa + 2 * MT * 512;
  const unsigned bar0 = smem_u32(tc_bar);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kTcMaxStages + s); };
  auto accf_bar = [&](int b) { return bar0 + 8u * (2 * kTcMaxStages + b); };
  auto acce_bar = [&](int b) { return bar0 + 8u * (2 * kTcMaxStages + 2 + b); };
  const unsigned drain_bar = bar0 + 8u * (2 * kTcMaxStages + 4);

  if (threadIdx.x == 0) {
    if (S < 2) set_error(a, kErrDevice);
    tc_run = S >= 2 && !failed(a);
    for (int s = 0; s < kTcMaxStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(smem_u32(&tc_tmem), kTcTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = tc_tmem;
  const bool run = tc_run != 0;
  // TMEM columns: D[buf][mt][half] at ((buf * MT + mt) * 2 + half) * 32, then per stage 4 columns per
  // scale block (SFA[mt][half], SFB)
  auto d_col = [&](int b, int mt, int h) { return (unsigned)(((b * MT + mt) * 2 + h) * 32); };
  auto sf_col = [&](int s, int i) { return tmem + (unsigned)(kTcDCols + (s * (2 * MT + 1) + i) * 4); };

  if ((warp == 0 || warp == 2) && run) {
    // ---- producers: warp 0 takes the even units and warp 2 the odd ones. Each gathers its units' weight
    // scales (through registers, D of its units ahead) and lane 0 then issues the unit's TMA / bulk copies.
    constexpr int D = 2;
    const int pw = warp >> 1;   // 0 or 1
    const unsigned long long pol = l2_evict_first_policy();
    const int sbytes = ph.K >> 5;
    unsigned sreg[D][MT][2][4];
    TcIter la = it0;   // look-ahead iterator (scales)
    if (pw) step(la);
    int la_chunk = -1;
    const uint8_t* la_scl[MT];
    auto load_scales = [&](unsigned (&r)[MT][2][4]) {
      if (la.chunk != la_chunk) {
        int e, fp, np;
        chunk_info(la.chunk, e, fp, np);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) la_scl[mt] = ph.scales[mt] + (size_t)e * ph.expert_scales;
        la_chunk = la.chunk;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int m1 = 0; m1 < 4; ++m1) {
          int row = la.tile * kTcRows + h * 128 + m1 * 32 + lane;
          row = row < ph.rows ? row : ph.rows - 1;   // rows past the matrix multiply zero codes
          const size_t off = (size_t)row * sbytes + la.ks * 4;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) r[mt][h][m1] = __ldg(reinterpret_cast<const unsigned*>(la_scl[mt] + off));
        }
      step(la);
      step(la);
    };
    const int mine = (nunits - pw + 1) >> 1;   // units pw, pw + 2, ...
#pragma unroll
    for (int d = 0; d < D; ++d)
      if (d < mine) load_scales(sreg[d]);
    TcIter it = it0;
    if (pw) step(it);
    int cur_chunk = -1, e = 0, p0 = 0, na = 1;
    bool ok = true;
    int last_i = -1;
    for (int k0 = 0; k0 < mine && ok; k0 += D) {
#pragma unroll
      for (int d = 0; d < D; ++d) {
        const int k = k0 + d;
        if (k >= mine) break;
        const int i = 2 * k + pw;
        const int s = i % S, round = i / S;
        if (round > 0 && !mbar_wait(a, empty_bar(s), (unsigned)(round - 1) & 1u)) {
          ok = false;
          break;
        }
        const unsigned st = base + (unsigned)s * stage_bytes;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(st + off_sfa + (mt * 2 + h) * 512 + lane * 16),
                         "r"(sreg[d][mt][h][0]), "r"(sreg[d][mt][h][1]), "r"(sreg[d][mt][h][2]), "r"(sreg[d][mt][h][3])
                         : "memory");
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (it.chunk != cur_chunk) {
            int fp, np;
            chunk_info(it.chunk, e, fp, np);
            p0 = fp & ~7;
            na = ((fp + np + 7) >> 3) - (p0 >> 3);
            cur_chunk = it.chunk;
          }
          mbar_arrive_tx(full_bar(s), MT * 16384u + (unsigned)na * 2304u);   // codes + 2 KB images + 256 B scales per atom
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
            tma_load_3d(st + mt * 32768, ph.map[mt], full_bar(s), it.ks * 128, it.tile * kTcRows, e, pol);
          const size_t atom0 = (size_t)it.ks * ph.atoms + (p0 >> 3);
          bulk_load(st + off_b, ph.bimg + (atom0 << 11), (unsigned)na << 11, full_bar(s));
          bulk_load(st + off_sfb, ph.bsfb + (atom0 << 8), (unsigned)na << 8, full_bar(s));
        }
        __syncwarp();
        last_i = i;
        if (k + D < mine) load_scales(sreg[d]);
        step(it);
        step(it);
      }
    }
    // every issued copy has landed before the CTA leaves (bounded): the last S units of the range are the last
    // use of their stages; each producer waits for the ones it issued
    if (lane == 0 && ok)
      for (int i = nunits - 1; i >= 0 && i >= nunits - S; --i)
        if ((i & 1) == pw && i <= last_i) mbar_wait(a, full_bar(i % S), (unsigned)(i / S) & 1u);
  } else if (warp == 1 && run) {
    // ---- MMA issuer (one thread)
    if (lane == 0) {
      unsigned accn[2] = {0u, 0u};
      int buf = 0;
      TcIter it = it0;
      int cur_chunk = -1, n = 16;
      unsigned idesc[4];
      int s = 0;
      unsigned ph_full = 0u;
      const unsigned long long dA = sdesc_sw128(base), dB = sdesc_sw128(base + off_b);
      const unsigned long long dSA = sdesc_rows16(base + off_sfa), dSB = sdesc_rows16(base + off_sfb);
      const unsigned long long stage_step = (unsigned long long)(stage_bytes >> 4);
      for (int i = 0; i < nunits; ++i) {
        const bool seg_first = i == 0 || it.ks == 0, seg_last = i == nunits - 1 || it.ks == ksteps - 1;
        if (it.chunk != cur_chunk) {
          int e, fp, np;
          chunk_info(it.chunk, e, fp, np);
          n = (((fp + np + 7) >> 3) - ((fp & ~7) >> 3)) * 8 * kTcTerms;
#pragma unroll
          for (int kb = 0; kb < 4; ++kb) idesc[kb] = idesc_mxf4_e4m3(n, (unsigned)kb);
          cur_chunk = it.chunk;
        }
        if (seg_first && accn[buf] > 0 && !mbar_wait(a, acce_bar(buf), (accn[buf] - 1) & 1u)) break;
        if (!mbar_wait(a, full_bar(s), ph_full)) break;
        tc_fence_after();
        const unsigned long long so = stage_step * (unsigned)s;
#pragma unroll
        for (int j = 0; j < 2 * MT; ++j) tmem_cp_32x128b_x4(sf_col(s, j), dSA + so + (unsigned)(j * 32));
        tmem_cp_32x128b_x4(sf_col(s, 2 * MT), dSB + so);
        const unsigned sfb = sf_col(s, 2 * MT);
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              umma_mxf8f6f4(tmem + d_col(buf, mt, h), dA + so + (unsigned)(mt * 2048 + h * 1024 + kb * 2),
                            dB + so + (unsigned)(kb * 2), idesc[kb], sf_col(s, mt * 2 + h) | ((unsigned)kb << 30),
                            sfb | ((unsigned)kb << 30), (seg_first && kb == 0) ? 0u : 1u);
        }
        umma_commit(empty_bar(s));
        if (seg_last) {
          umma_commit(accf_bar(buf));
          ++accn[buf];
          buf ^= 1;
        }
        step(it);
        if (++s == S) {
          s = 0;
          ph_full ^= 1u;
        }
      }
    }
  } else if (warp >= 4 && warp < 4 + kEpiWarps && run) {
    // ---- epilogue: warp 4 + 4h + q reads TMEM lanes 32q..32q+31 of half h = tile rows 128h + 32q + lane
    const int h = (warp - 4) >> 2, q = (warp - 4) & 3, row = 128 * h + 32 * q + lane;
    const unsigned lane_base = (unsigned)(32 * q) << 16;
    unsigned accn[2] = {0u, 0u};
    int buf = 0;
    int i = 0;
    TcIter it = it0;
    while (i < nunits) {
      const int chunk = it.chunk, tile = it.tile, ks = it.ks;
      const int seg_len = (ksteps - ks) < (nunits - i) ? (ksteps - ks) : (nunits - i);
      const bool whole = ks == 0 && seg_len == ksteps;
      int e, fp, np;
      chunk_info(chunk, e, fp, np);
      if (!mbar_wait(a, accf_bar(buf), accn[buf] & 1u)) break;
      ++accn[buf];
      tc_fence_after();
      // pair j of the chunk is row r = fp + j - p0 of the window: columns (r / 8) * 16 + t * 8 + r % 8
      const int p0 = fp & ~7;
      float v[MT][8];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int r = fp + (j < np ? j : 0) - p0;
          const unsigned c = tmem + lane_base + d_col(buf, mt, h) + (unsigned)((r >> 3) * 16 + (r & 7));
          v[mt][j] = tmem_ld1(c) + tmem_ld1(c + 8);
        }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(buf));
      buf ^= 1;
      bool fin = whole;
      if (!whole) {
        // stream-K: publish this CTA's partial, the last contributor to arrive finishes the tile
        const int tile_beg = chunk * per_chunk + tile * ksteps;
        const int first = (int)owner_of(tile_beg, U, G), last = (int)owner_of(tile_beg + ksteps - 1, U, G);
        const int slot = ubeg >= tile_beg ? 0 : 1;
        float* mine = ph.part + ((size_t)blockIdx.x * 2 + slot) * (MT * 8 * kTcRows);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int j = 0; j < 8; ++j) __stcg(mine + (mt * 8 + j) * kTcRows + row, v[mt][j]);
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        if (h == 0 && q == 0 && lane == 0) {
          int* c = ph.cnt + chunk * tiles + tile;
          const int old = atom_add_acq_rel_gpu(c, 1);
          const int lastp = old == last - first;
          if (lastp) *c = 0;
          tc_last = lastp;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
        fin = tc_last != 0;
        if (fin) {
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 8; ++j) v[mt][j] = 0.0f;
          for (int cta = first; cta <= last; ++cta) {
            const int cbeg = (int)((long long)U * cta / G);
            const float* src = ph.part + ((size_t)cta * 2 + (cbeg >= tile_beg ? 0 : 1)) * (MT * 8 * kTcRows);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
              for (int j = 0; j < 8; ++j) v[mt][j] += __ldcg(src + (mt * 8 + j) * kTcRows + row);
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");   // tc_last is rewritten by the next split tile
      }
      const int orow = tile * kTcRows + row;   // output row of the matrix (inter row or latent row)
      if (fin && orow < ph.rows) {
        if (MT == 2) {
          // activations of the down projection: bf16-rounded situ(gate, up), quantised over the warp's
          // 32 rows (one k-block of the down projection's k-step orow / 128)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j >= np) break;   // np is uniform across the warp
            const int p = fp + j;
            const float act = round_bf(situ_f(round_bf(v[0][j]), round_bf(v[MT - 1][j])));
            tc_store_terms(ph.oimg, ph.osfb, ph.atoms, orow >> 7, p, orow & 127, act);
            if (ph.act_dbg) ph.act_dbg[(size_t)p * ph.rows + orow] = __float2half_rn(act);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (j >= np) break;
            const int p = fp + j;
            int b = __ldcg(a.s.pair_row + p), slot = __ldcg(a.s.pair_slot + p);
            b = b < 0 ? 0 : (b >= a.g.B ? a.g.B - 1 : b);
            slot = slot < 0 ? 0 : (slot >= a.g.K ? a.g.K - 1 : slot);
            a.s.out_slot[((size_t)b * a.g.K + slot) * a.g.lh + orow] = f2bf(v[0][j]);
          }
        }
      }
      i += seg_len;
      for (int k = 0; k < seg_len; ++k) step(it);
    }
  }
  // drain: the issuer waits until every MMA and scale copy it issued has completed; then TMEM is freed
  if (warp == 1 && lane == 0 && run) {
    umma_commit(drain_bar);
    mbar_wait(a, drain_bar, 0u);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  __syncwarp();
  if (warp == 1) tmem_dealloc(tmem, kTcTmemCols);
  if (threadIdx.x == 0)
    for (int s = 0; s < kTcBars; ++s) mbar_inval(bar0 + 8u * s);
}

}  // namespace kk3
