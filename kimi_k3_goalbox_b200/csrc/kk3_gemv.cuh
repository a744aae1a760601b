// kk3_gemv.cuh - weight-streaming matrix-vector products on sm_100a tensor cores (mma.sync m16n8k16).
//
// Every projection of the decode step is y[b, n] = sum_k x[b, k] * W[n, k] with a weight matrix W that is
// read exactly once per step from HBM and a tiny batch of activations x (B <= 64). The weight rows are the
// M dimension of the MMA (16-row tiles), the batch is N (8 columns per n-tile), FP32 accumulation.
//
// Work split: "warp-level stream-K". A phase's units are (16-row tile, 64-wide k-step) pairs over all of its
// jobs. Every warp of the grid gets one contiguous, equally long range of units, so the HBM stream is
// balanced to one k-step regardless of matrix shapes. A tile whose units span several warps is finished by
// the last warp to arrive (per-tile arrival counter): it adds the partial tiles of the other warps in warp
// order, so results are deterministic and identical on every rank (replicated projections such as the
// router must agree bit for bit across tensor-parallel ranks). The finishing warp runs the fused epilogue
// (BF16 rounding where the reference rounds, sigmoid, SiLU-like `situ`, argmax keys, peer exchange stores).
//
// Weights are permuted along k in registers: lane (r = lane/4, c = lane%4) loads 16 contiguous bytes of rows
// r and r+8 at k = 64s + 8c and 64s + 32 + 8c, so one warp load covers 64 contiguous bytes per row; the
// activation operand is read with the same permutation, which leaves the dot product unchanged.
#pragma once

#include "kk3_common.cuh"

namespace kk3 {

enum Epi : int {
  EPI_STORE_BF16 = 0,   // out bf16 [col, ldo]
  EPI_SIGMOID_F32,      // out f32 [col, ldo] = sigmoid(acc)         (router scores, kimi.py:308)
  EPI_SITU,             // dual job: out bf16 = situ(bf16 gate, bf16 up) (kimi.py:194-196, :304, :326)
  EPI_LATENT,           // out bf16 [col, ldo] and out2 f16 permuted copy for the MXFP4 path
  EPI_LOGITS,           // out f32 [col, ldo] = bf16-rounded logits, argmax keys (kimi.py:331, :218-227)
  EPI_ROUTED,           // prefix[col, row] += bf16(bf16(acc) + shared_red[col, row]) (kimi.py:325-329)
  EPI_EXCHANGE,         // bf16(acc) into every rank's exchange region [src][col][row] (kimi.py:343-347)
};

struct GemvJob {
  const bf16* w;        // weights [rows, K] (row-major, K contiguous)
  const bf16* w2;       // second matrix of a dual job (the `up` projection), same shape
  const bf16* x;        // activations [ncols, ldx]
  void* out;
  void* out2;
  const void* aux;
  long long ubase;      // first unit of this job in the phase's unit space
  int rows, K, ldx, ncols, ldo, epi, tiles, ksteps, tile0;
  long long aux_off;    // epilogue extra (exchange sub-region offset, vocab offset, ...)
};

constexpr int kMaxJobs = 8;

KK3_DEV long long owner_of(long long u, long long U, long long GW) { return ((u + 1) * GW - 1) / U; }

template <int NT, int MT>
KK3_DEV void mma_rows_bf16(const bf16* const (&wa)[MT], const bf16* const (&wb)[MT], const bf16* __restrict__ x,
                           int ldx, int ncols, int ks0, int ks1, float (&acc)[MT][NT][4]) {
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const bf16* xr[NT];
  bool xv[NT];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n = nt * 8 + r;
    xv[nt] = n < ncols;
    xr[nt] = x + (size_t)(xv[nt] ? n : 0) * ldx + 8 * c;
  }
  constexpr int kUnroll = (NT * MT <= 2) ? 4 : ((NT * MT <= 4) ? 2 : 1);
#pragma unroll kUnroll
  for (int ks = ks0; ks < ks1; ++ks) {
    const int k0 = ks * 64 + 8 * c;
    uint4 A0[MT], A1[MT], B0[MT], B1[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      A0[mt] = ldg_stream16(wa[mt] + k0);
      A1[mt] = ldg_stream16(wa[mt] + k0 + 32);
      B0[mt] = ldg_stream16(wb[mt] + k0);
      B1[mt] = ldg_stream16(wb[mt] + k0 + 32);
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
      if (xv[nt]) {
        X0 = ld_act16(xr[nt] + ks * 64);
        X1 = ld_act16(xr[nt] + ks * 64 + 32);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        mma_bf16(acc[mt][nt], A0[mt].x, B0[mt].x, A0[mt].y, B0[mt].y, X0.x, X0.y);
        mma_bf16(acc[mt][nt], A0[mt].z, B0[mt].z, A0[mt].w, B0[mt].w, X0.z, X0.w);
        mma_bf16(acc[mt][nt], A1[mt].x, B1[mt].x, A1[mt].y, B1[mt].y, X1.x, X1.y);
        mma_bf16(acc[mt][nt], A1[mt].z, B1[mt].z, A1[mt].w, B1[mt].w, X1.z, X1.w);
      }
    }
  }
}

KK3_DEV float situ_f(float g, float u) {
  return 4.0f * tanhf(g / 4.0f) * sigmoidf_(g) * (25.0f * tanhf(u / 25.0f));
}

KK3_DEV unsigned long long argmax_key(float v, unsigned idx) {
  unsigned b = __float_as_uint(v);
  unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (unsigned long long)(0xffffffffu - idx);
}

// exchange region of rank `dst` as seen from this rank, parity p
KK3_DEV unsigned char* xregion(const StepArgs& a, int dst, int parity) {
  return a.comm.base[dst] + a.comm.data_off[parity];
}

// Fused epilogue for one complete 16-row tile. acc[mt][nt][i]: rows row0 + r (+8 for i >= 2), column
// nt*8 + 2c + (i & 1).
template <int NT, int MT>
KK3_DEV void gemv_epilogue(const StepArgs& a, const GemvJob& j, int tile, const float (&acc)[MT][NT][4], int parity) {
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const int row0 = tile * 16;
  if (j.epi == EPI_LOGITS) {
    // per-column max over the tile's rows, lowest index on ties, then one atomicMax per column
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = nt * 8 + 2 * c + e;
        unsigned long long best = 0ull;
#pragma unroll
        for (int hi = 0; hi < 2; ++hi) {
          const int row = row0 + r + 8 * hi;
          if (row < j.rows && col < j.ncols) {
            const float v = round_bf(acc[0][nt][hi * 2 + e]);
            reinterpret_cast<float*>(j.out)[(size_t)col * j.ldo + row] = v;
            const unsigned long long k = argmax_key(v, (unsigned)(row + j.aux_off));
            best = k > best ? k : best;
          }
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
          best = other > best ? other : best;
        }
        if (r == 0 && col < j.ncols && best != 0ull)
          atomicMax(reinterpret_cast<unsigned long long*>(const_cast<void*>(j.aux)) + col, best);
      }
    }
    return;
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = row0 + r + 8 * (i >> 1);
      const int col = nt * 8 + 2 * c + (i & 1);
      if (row >= j.rows || col >= j.ncols) continue;
      const float v = acc[0][nt][i];
      const size_t o = (size_t)col * j.ldo + row;
      switch (j.epi) {
        case EPI_STORE_BF16:
          reinterpret_cast<bf16*>(j.out)[o] = f2bf(v);
          break;
        case EPI_SIGMOID_F32:
          reinterpret_cast<float*>(j.out)[o] = sigmoidf_(v);
          break;
        case EPI_SITU: {
          const float g = round_bf(v), u = round_bf(acc[MT - 1][nt][i]);
          reinterpret_cast<bf16*>(j.out)[o] = f2bf(situ_f(g, u));
          break;
        }
        case EPI_LATENT: {
          const bf16 b = f2bf(v);
          reinterpret_cast<bf16*>(j.out)[o] = b;
          reinterpret_cast<__half*>(j.out2)[(size_t)col * j.ldo + perm8(row)] = __float2half_rn(bf2f(b));
          break;
        }
        case EPI_ROUTED: {
          bf16* prefix = reinterpret_cast<bf16*>(j.out);
          const bf16* shared = reinterpret_cast<const bf16*>(j.aux);
          const float out = round_bf(round_bf(v) + bf2f(shared[o]));
          prefix[o] = f2bf(bf2f(prefix[o]) + out);
          break;
        }
        case EPI_EXCHANGE: {
          // layout [src][col][ldo], src = this rank; written into every rank's region
          const bf16 b = f2bf(v);
          const size_t off = (size_t)a.g.rank * a.g.B * j.ldo + o;
          for (int dst = 0; dst < a.g.tp; ++dst)
            reinterpret_cast<bf16*>(xregion(a, dst, parity) + j.aux_off)[off] = b;
          break;
        }
        default:
          break;
      }
    }
  }
}

// Run a list of dense BF16 jobs with warp-level stream-K over CTAs [cta_lo, cta_hi).
template <int NT, int MT>
KK3_DEV void run_gemv(const StepArgs& a, const GemvJob* jobs, int njobs, int cta_lo, int cta_hi, int parity,
                         int bank = 0) {
  if ((int)blockIdx.x < cta_lo || (int)blockIdx.x >= cta_hi) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2;
  const GemvJob& last = jobs[njobs - 1];
  const long long U = last.ubase + (long long)last.tiles * last.ksteps;
  long long GW = (long long)(cta_hi - cta_lo) * kWarps;
  GW = GW < U ? GW : U;
  const long long gw = (long long)(blockIdx.x - cta_lo) * kWarps + warp;
  if (U == 0 || gw >= GW) return;
  const long long ubeg = U * gw / GW, uend = U * (gw + 1) / GW;
  constexpr int kSlot = MT * NT * 128;   // floats per partial tile
  float* my_slot0 = a.s.fix_part + bank * a.g.fix_bank + (size_t)(gw * 2) * kSlot;
  int ji = 0;
  for (long long u = ubeg; u < uend;) {
    while (u >= jobs[ji].ubase + (long long)jobs[ji].tiles * jobs[ji].ksteps) ++ji;
    const GemvJob& j = jobs[ji];
    const long long local = u - j.ubase;
    const int tile = (int)(local / j.ksteps);
    const int ks0 = (int)(local % j.ksteps);
    const long long tile_beg = j.ubase + (long long)tile * j.ksteps, tile_end = tile_beg + j.ksteps;
    const long long seg_end = uend < tile_end ? uend : tile_end;
    const int ks1 = ks0 + (int)(seg_end - u);

    const bf16* wa[MT];
    const bf16* wb[MT];
    {
      int ra = tile * 16 + r, rb = ra + 8;
      ra = ra < j.rows ? ra : j.rows - 1;
      rb = rb < j.rows ? rb : j.rows - 1;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const bf16* base = (mt == 0) ? j.w : j.w2;
        wa[mt] = base + (size_t)ra * j.K;
        wb[mt] = base + (size_t)rb * j.K;
      }
    }
    float acc[MT][NT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.0f;
    mma_rows_bf16<NT, MT>(wa, wb, j.x, j.ldx, j.ncols, ks0, ks1, acc);

    const long long first = owner_of(tile_beg, U, GW), lastw = owner_of(tile_end - 1, U, GW);
    if (first == lastw) {
      gemv_epilogue<NT, MT>(a, j, tile, acc, parity);
    } else {
      float* slot = my_slot0 + (u == ubeg ? 0 : kSlot);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) slot[((mt * NT + nt) * 4 + i) * 32 + lane] = acc[mt][nt][i];
      __threadfence();
      __syncwarp();
      int old = 0;
      if (lane == 0) old = atomicAdd(a.s.fix_cnt + bank * a.g.cnt_bank + j.tile0 + tile, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == (int)(lastw - first)) {
        __threadfence();
        float sum[MT][NT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) sum[mt][nt][i] = 0.0f;
        for (long long w = first; w <= lastw; ++w) {
          if (w == gw) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) sum[mt][nt][i] += acc[mt][nt][i];
          } else {
            const long long wbeg = U * w / GW;
            const float* ps = a.s.fix_part + bank * a.g.fix_bank + (size_t)(w * 2 + (wbeg >= tile_beg ? 0 : 1)) * kSlot;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
              for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) sum[mt][nt][i] += ld_cg_f32(ps + ((mt * NT + nt) * 4 + i) * 32 + lane);
          }
        }
        gemv_epilogue<NT, MT>(a, j, tile, sum, parity);
        if (lane == 0) atomicExch(a.s.fix_cnt + bank * a.g.cnt_bank + j.tile0 + tile, 0);
      }
    }
    u = seg_end;
  }
}

// Finalise job unit bases / tile counts (all threads compute identical values).
KK3_DEV void prepare_jobs(GemvJob* jobs, int njobs) {
  long long ub = 0;
  int t0 = 0;
  for (int i = 0; i < njobs; ++i) {
    jobs[i].tiles = (jobs[i].rows + 15) / 16;
    jobs[i].ksteps = jobs[i].K / 64;
    jobs[i].ubase = ub;
    jobs[i].tile0 = t0;
    ub += (long long)jobs[i].tiles * jobs[i].ksteps;
    t0 += jobs[i].tiles;
  }
}

// ------------------------------------------------------------------------------------------------
// MXFP4 routed experts (e2m1 codes [rows, K/32, 16] + E8M0 scales [rows, K/32], kimi.py:116-119).
// One n-tile of <= 8 (expert, token) pairs per unit; the 32-wide scale groups are applied to the FP32
// accumulator exactly (one zero-initialised 2-step MMA per group, then acc += t * 2^(s-127)).

template <int MT>
KK3_DEV void mma_rows_fp4(const uint8_t* const (&ca)[MT], const uint8_t* const (&cb)[MT],
                          const uint8_t* const (&sa)[MT], const uint8_t* const (&sb)[MT],
                          const __half* xrow, int ks0, int ks1, float (&acc)[MT][4]) {
  const int lane = threadIdx.x & 31, c = lane & 3;
#pragma unroll 2
  for (int g = ks0 * 2; g < ks1 * 2; ++g) {
    uint4 X = make_uint4(0, 0, 0, 0);
    if (xrow) X = ld_act16(xrow + g * 32 + 8 * c);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const unsigned wa = ldg_nc32(ca[mt] + g * 16 + 4 * c);
      const unsigned wb = ldg_nc32(cb[mt] + g * 16 + 4 * c);
      const float fa = e8m0_to_f32(ldg_nc8(sa[mt] + g));
      const float fb = e8m0_to_f32(ldg_nc8(sb[mt] + g));
      unsigned ra[4], rb[4];
      e2m1x8_to_f16(wa, ra);
      e2m1x8_to_f16(wb, rb);
      float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      mma_f16(t, ra[0], rb[0], ra[1], rb[1], X.x, X.y);
      mma_f16(t, ra[2], rb[2], ra[3], rb[3], X.z, X.w);
      acc[mt][0] = fmaf(t[0], fa, acc[mt][0]);
      acc[mt][1] = fmaf(t[1], fa, acc[mt][1]);
      acc[mt][2] = fmaf(t[2], fb, acc[mt][2]);
      acc[mt][3] = fmaf(t[3], fb, acc[mt][3]);
    }
  }
}

struct ExpertPhase {
  const uint8_t* codes[2];   // gate/up blocks (MT=2) or down blocks (MT=1), expert 0
  const uint8_t* scales[2];
  int rows, K;               // per expert: rows of the matrix, inner dimension
  int tiles, ksteps;
  long long expert_codes;    // bytes of codes per expert (rows * K / 2)
  long long expert_scales;   // bytes of scales per expert (rows * K / 32)
};

template <int MT>
KK3_DEV void expert_epilogue(const StepArgs& a, const ExpertPhase& ph, int first_pair, int npairs, int tile,
                             const float (&acc)[MT][4]) {
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = tile * 16 + r + 8 * (i >> 1);
    const int col = 2 * c + (i & 1);
    if (col >= npairs || row >= ph.rows) continue;
    const int p = first_pair + col;
    if (MT == 2) {
      const float g = round_bf(acc[0][i]), u = round_bf(acc[MT - 1][i]);
      const float act = round_bf(situ_f(g, u));
      a.s.act_p[(size_t)p * a.g.inter + perm8(row)] = __float2half_rn(act);
    } else {
      int b = a.s.pair_row[p], slot = a.s.pair_slot[p];
      b = b < 0 ? 0 : (b >= a.g.B ? a.g.B - 1 : b);
      slot = slot < 0 ? 0 : (slot >= a.g.K ? a.g.K - 1 : slot);
      a.s.out_slot[((size_t)b * a.g.K + slot) * a.g.lh + row] = f2bf(acc[0][i]);
    }
  }
}

// Stream-K over (expert chunk, tile, k-step) units. Chunks come from the routing phase.
template <int MT>
KK3_DEV void run_experts(const StepArgs& a, const ExpertPhase& ph) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2;
  int nchunks = ld_volatile_int(a.s.chunk_info);
  nchunks = nchunks < 0 ? 0 : (nchunks > a.g.B * a.g.K ? a.g.B * a.g.K : nchunks);
  const long long per_chunk = (long long)ph.tiles * ph.ksteps;
  const long long U = (long long)nchunks * per_chunk;
  if (U == 0) return;
  long long GW = (long long)gridDim.x * kWarps;
  GW = GW < U ? GW : U;
  const long long gw = (long long)blockIdx.x * kWarps + warp;
  if (gw >= GW) return;
  const long long ubeg = U * gw / GW, uend = U * (gw + 1) / GW;
  constexpr int kSlot = MT * 128;
  float* my_slot0 = a.s.fix_part + (size_t)(gw * 2) * kSlot;
  for (long long u = ubeg; u < uend;) {
    const int chunk = (int)(u / per_chunk);
    const long long local = u - (long long)chunk * per_chunk;
    const int tile = (int)(local / ph.ksteps);
    const int ks0 = (int)(local % ph.ksteps);
    const long long tile_beg = (long long)chunk * per_chunk + (long long)tile * ph.ksteps;
    const long long tile_end = tile_beg + ph.ksteps;
    const long long seg_end = uend < tile_end ? uend : tile_end;
    const int ks1 = ks0 + (int)(seg_end - u);
    // routing-table values are clamped so that a routing fault can never address outside the buffers
    const int npk = a.g.B * a.g.K;
    int expert = a.s.chunk_info[1 + chunk * 3];
    int first_pair = a.s.chunk_info[2 + chunk * 3];
    int npairs = a.s.chunk_info[3 + chunk * 3];
    expert = expert < 0 ? 0 : (expert >= a.g.E ? a.g.E - 1 : expert);
    first_pair = first_pair < 0 ? 0 : (first_pair >= npk ? npk - 1 : first_pair);
    npairs = npairs < 0 ? 0 : (npairs > 8 ? 8 : npairs);
    npairs = first_pair + npairs > npk ? npk - first_pair : npairs;

    const uint8_t* ca[MT];
    const uint8_t* cb[MT];
    const uint8_t* sa[MT];
    const uint8_t* sb[MT];
    {
      const int ra = tile * 16 + r, rb = ra + 8;   // rows are multiples of 16 for expert matrices
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint8_t* cbase = ph.codes[mt] + (size_t)expert * ph.expert_codes;
        const uint8_t* sbase = ph.scales[mt] + (size_t)expert * ph.expert_scales;
        ca[mt] = cbase + (size_t)ra * (ph.K / 2);
        cb[mt] = cbase + (size_t)rb * (ph.K / 2);
        sa[mt] = sbase + (size_t)ra * (ph.K / 32);
        sb[mt] = sbase + (size_t)rb * (ph.K / 32);
      }
    }
    const __half* xrow = nullptr;
    if (r < npairs) {
      const int p = first_pair + r;
      int prow = a.s.pair_row[p];
      prow = prow < 0 ? 0 : (prow >= a.g.B ? a.g.B - 1 : prow);
      xrow = (MT == 2) ? a.s.latent_p + (size_t)prow * a.g.lh : a.s.act_p + (size_t)p * a.g.inter;
    }
    float acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][i] = 0.0f;
    mma_rows_fp4<MT>(ca, cb, sa, sb, xrow, ks0, ks1, acc);

    const long long first = owner_of(tile_beg, U, GW), lastw = owner_of(tile_end - 1, U, GW);
    const int gtile = chunk * ph.tiles + tile;
    if (first == lastw) {
      expert_epilogue<MT>(a, ph, first_pair, npairs, tile, acc);
    } else {
      float* slot = my_slot0 + (u == ubeg ? 0 : kSlot);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) slot[(mt * 4 + i) * 32 + lane] = acc[mt][i];
      __threadfence();
      __syncwarp();
      int old = 0;
      if (lane == 0) old = atomicAdd(a.s.fix_cnt + gtile, 1);
      old = __shfl_sync(0xffffffffu, old, 0);
      if (old == (int)(lastw - first)) {
        __threadfence();
        float sum[MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int i = 0; i < 4; ++i) sum[mt][i] = 0.0f;
        for (long long w = first; w <= lastw; ++w) {
          if (w == gw) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
              for (int i = 0; i < 4; ++i) sum[mt][i] += acc[mt][i];
          } else {
            const long long wbeg = U * w / GW;
            const float* ps = a.s.fix_part + (size_t)(w * 2 + (wbeg >= tile_beg ? 0 : 1)) * kSlot;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
              for (int i = 0; i < 4; ++i) sum[mt][i] += ld_cg_f32(ps + (mt * 4 + i) * 32 + lane);
          }
        }
        expert_epilogue<MT>(a, ph, first_pair, npairs, tile, sum);
        if (lane == 0) atomicExch(a.s.fix_cnt + gtile, 0);
      }
    }
    u = seg_end;
  }
}

}  // namespace kk3
