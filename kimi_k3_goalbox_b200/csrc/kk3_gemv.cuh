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
// Weights are permuted along k in registers: lane (r = lane/4, c = lane%4) owns 16 contiguous bytes of rows
// r and r+8 at k = 64s + 8c and 64s + 32 + 8c, so one warp covers 64 contiguous bytes per row; the
// activation operand is read with the same permutation, which leaves the dot product unchanged.
// Bytes in flight: every warp streams its unit range through a private ring of cp.async stages in shared
// memory (6 k-steps deep, 2 KB each), so ~190 KB per SM are outstanding without holding registers; the
// producer cursor runs continuously across tile boundaries.
#pragma once

#include "kk3_common.cuh"

namespace kk3 {

enum Epi : int {
  EPI_STORE_BF16 = 0,   // out bf16 [col, ldo]
  EPI_SIGMOID_F32,      // out f32 [col, ldo] = sigmoid(acc)         (router scores, kimi.py:308)
  EPI_SITU,             // dual job: out bf16 = situ(bf16 gate, bf16 up) (kimi.py:194-196, :304, :326)
  EPI_LATENT,           // out bf16 [col, ldo] and out2 an FP16 copy for the MXFP4 path
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

KK3_DEV void cp_async16_g(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem_dst)),
               "l"(src) : "memory");
}
KK3_DEV void cp_async_commit_g() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
KK3_DEV void cp_async_wait_g() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One 64-wide k-step of a 16-row tile: A fragments from this lane's ring slot, activations from global.
template <int NT, int MT>
KK3_DEV void mma_step_bf16(const uint4* __restrict__ slot, const bf16* __restrict__ x, int ldx, int ncols, int ks,
                           float (&acc)[MT][NT][4]) {
  const int lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  uint4 A0[MT], A1[MT], B0[MT], B1[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    A0[mt] = slot[(mt * 4 + 0) * 32 + lane];
    A1[mt] = slot[(mt * 4 + 1) * 32 + lane];
    B0[mt] = slot[(mt * 4 + 2) * 32 + lane];
    B1[mt] = slot[(mt * 4 + 3) * 32 + lane];
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int n = nt * 8 + r;
    uint4 X0 = make_uint4(0, 0, 0, 0), X1 = make_uint4(0, 0, 0, 0);
    if (n < ncols) {
      const bf16* xr = x + (size_t)n * ldx + ks * 64 + 8 * c;
      X0 = ld_act16(xr);
      X1 = ld_act16(xr + 32);
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
          reinterpret_cast<__half*>(j.out2)[(size_t)col * j.ldo + row] = __float2half_rn(bf2f(b));
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

// Deterministic combination of a tile split over warps first..lastw (see the file comment). `acc` is this
// warp's partial; slot 0/1 of a warp holds its first/other partial tile. Returns true (with the complete
// tile in `acc`) when this warp arrived last and must run the epilogue.
template <int NV>
KK3_DEV bool stream_k_fixup(const StepArgs& a, float* part_base, int* cnt, long long gw, bool first_seg,
                            long long tile_beg, long long first, long long lastw, long long U, long long GW,
                            float (&acc)[NV]) {
  const int lane = threadIdx.x & 31;
  float* slot = part_base + (size_t)(gw * 2 + (first_seg ? 0 : 1)) * (NV * 32);
#pragma unroll
  for (int i = 0; i < NV; ++i) slot[i * 32 + lane] = acc[i];
  __threadfence();
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atomicAdd(cnt, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != (int)(lastw - first)) return false;
  __threadfence();
  float sum[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) sum[i] = 0.0f;
  for (long long w = first; w <= lastw; ++w) {
    if (w == gw) {
#pragma unroll
      for (int i = 0; i < NV; ++i) sum[i] += acc[i];
    } else {
      const long long wbeg = U * w / GW;
      const float* ps = part_base + (size_t)(w * 2 + (wbeg >= tile_beg ? 0 : 1)) * (NV * 32);
#pragma unroll
      for (int i = 0; i < NV; ++i) sum[i] += ld_cg_f32(ps + i * 32 + lane);
    }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) acc[i] = sum[i];
  if (lane == 0) atomicExch(cnt, 0);
  return true;
}

// position of a unit in a job list
struct Cursor {
  int ji, tile, ks;
};

KK3_DEV Cursor locate(const GemvJob* jobs, long long u) {
  Cursor c;
  c.ji = 0;
  while (u >= jobs[c.ji].ubase + (long long)jobs[c.ji].tiles * jobs[c.ji].ksteps) ++c.ji;
  const long long local = u - jobs[c.ji].ubase;
  c.tile = (int)(local / jobs[c.ji].ksteps);
  c.ks = (int)(local % jobs[c.ji].ksteps);
  return c;
}

KK3_DEV void advance(Cursor& c, const GemvJob* jobs) {
  if (++c.ks == jobs[c.ji].ksteps) {
    c.ks = 0;
    if (++c.tile == jobs[c.ji].tiles) {
      c.tile = 0;
      ++c.ji;
    }
  }
}

// stage this lane's 16-byte pieces of one unit (rows r, r+8; k = 64ks + 8c and +32) into its ring slot
template <int MT>
KK3_DEV void issue_bf16(const GemvJob& j, const Cursor& c, uint4* slot) {
  const int lane = threadIdx.x & 31, r = lane >> 2, cc = lane & 3;
  int ra = c.tile * 16 + r, rb = ra + 8;
  ra = ra < j.rows ? ra : j.rows - 1;
  rb = rb < j.rows ? rb : j.rows - 1;
  const int k0 = c.ks * 64 + 8 * cc;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const bf16* base = (mt == 0) ? j.w : j.w2;
    const bf16* pa = base + (size_t)ra * j.K + k0;
    const bf16* pb = base + (size_t)rb * j.K + k0;
    cp_async16_g(slot + (mt * 4 + 0) * 32 + lane, pa);
    cp_async16_g(slot + (mt * 4 + 1) * 32 + lane, pa + 32);
    cp_async16_g(slot + (mt * 4 + 2) * 32 + lane, pb);
    cp_async16_g(slot + (mt * 4 + 3) * 32 + lane, pb + 32);
  }
}

constexpr int kGemvSmemPerWarp = 12 * 1024;   // ring bytes per warp (6 stages x 2 KB, or 3 x 4 KB)

// Run a list of dense BF16 jobs with warp-level stream-K over CTAs [cta_lo, cta_hi).
template <int NT, int MT>
KK3_DEV void run_gemv(const StepArgs& a, const GemvJob* jobs, int njobs, int cta_lo, int cta_hi, int parity,
                         int bank = 0) {
  if ((int)blockIdx.x < cta_lo || (int)blockIdx.x >= cta_hi) return;
  extern __shared__ __align__(16) unsigned char kk3_dyn_smem[];
  constexpr int S = (MT == 1) ? 6 : 3;   // ring depth in units
  constexpr int kSlotVec = MT * 4 * 32;  // uint4 per unit slot
  const int warp = threadIdx.x >> 5;
  const GemvJob& lastj = jobs[njobs - 1];
  const long long U = lastj.ubase + (long long)lastj.tiles * lastj.ksteps;
  long long GW = (long long)(cta_hi - cta_lo) * kWarps;
  GW = GW < U ? GW : U;
  const long long gw = (long long)(blockIdx.x - cta_lo) * kWarps + warp;
  if (U == 0 || gw >= GW) return;
  const long long ubeg = U * gw / GW, uend = U * (gw + 1) / GW;
  uint4* ring = reinterpret_cast<uint4*>(kk3_dyn_smem + (size_t)warp * kGemvSmemPerWarp);
  float* part_base = a.s.fix_part + bank * a.g.fix_bank;
  int* cnt_base = a.s.fix_cnt + bank * a.g.cnt_bank;

  Cursor pc = locate(jobs, ubeg);
  Cursor cc = pc;
  long long pu = ubeg;
#pragma unroll
  for (int i = 0; i < S - 1; ++i) {
    if (pu < uend) {
      issue_bf16<MT>(jobs[pc.ji], pc, ring + (int)((pu - ubeg) % S) * kSlotVec);
      advance(pc, jobs);
      ++pu;
    }
    cp_async_commit_g();
  }
  float acc[MT][NT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.0f;
  long long seg_start = ubeg;
  for (long long u = ubeg; u < uend; ++u) {
    if (pu < uend) {
      issue_bf16<MT>(jobs[pc.ji], pc, ring + (int)((pu - ubeg) % S) * kSlotVec);
      advance(pc, jobs);
      ++pu;
    }
    cp_async_commit_g();
    cp_async_wait_g<S - 1>();
    const GemvJob& j = jobs[cc.ji];
    mma_step_bf16<NT, MT>(ring + (int)((u - ubeg) % S) * kSlotVec, j.x, j.ldx, j.ncols, cc.ks, acc);
    if (cc.ks == j.ksteps - 1 || u == uend - 1) {
      const long long tile_beg = j.ubase + (long long)cc.tile * j.ksteps;
      const long long first = owner_of(tile_beg, U, GW), lastw = owner_of(tile_beg + j.ksteps - 1, U, GW);
      bool done = first == lastw;
      if (!done) {
        done = stream_k_fixup<MT * NT * 4>(a, part_base, cnt_base + j.tile0 + cc.tile, gw, seg_start == ubeg,
                                           tile_beg, first, lastw, U, GW,
                                           *reinterpret_cast<float(*)[MT * NT * 4]>(&acc[0][0][0]));
      }
      if (done) gemv_epilogue<NT, MT>(a, j, cc.tile, acc, parity);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.0f;
      seg_start = u + 1;
    }
    advance(cc, jobs);
  }
  cp_async_wait_g<0>();
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
      a.s.act_p[(size_t)p * a.g.inter + row] = __float2half_rn(act);
    } else {
      int b = a.s.pair_row[p], slot = a.s.pair_slot[p];
      b = b < 0 ? 0 : (b >= a.g.B ? a.g.B - 1 : b);
      slot = slot < 0 ? 0 : (slot >= a.g.K ? a.g.K - 1 : slot);
      a.s.out_slot[((size_t)b * a.g.K + slot) * a.g.lh + row] = f2bf(acc[0][i]);
    }
  }
}

// E2M1 pairs -> FP16 pairs with the sm_100a hardware conversion: byte j of w -> register j holding
// (low nibble, high nibble) = elements (2j, 2j+1).
KK3_DEV void e2m1x8_cvt(unsigned w, unsigned (&r)[4]) {
  asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %4;\n"
      " cvt.rn.f16x2.e2m1x2 %0, b0;\n cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      " cvt.rn.f16x2.e2m1x2 %2, b2;\n cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(w));
}

KK3_DEV unsigned lds32(const unsigned char* p) { return *reinterpret_cast<const unsigned*>(p); }

constexpr int kFp4Row = 48;                 // staged bytes per row and unit (32 used; 48 keeps LDS conflict-free)
constexpr int kFp4Slot = 16 * kFp4Row;      // one matrix, one unit

struct ExpertCursor {
  int chunk, tile, ks;
};

// Stream-K over (expert chunk, tile, k-step) units. Chunks come from the routing phase. A unit is a
// 16-row tile x 64 k (two E2M1 groups); the warp's 32 lanes stage its 16 rows x 32 bytes per matrix with
// one 16-byte cp.async each into a ring (8 deep for gate+up, 16 for down), then every quad reads its
// rows' 4-byte quarters, converts E2M1 -> FP16 in hardware, and applies the E8M0 scale per group in FP32.
template <int MT>
KK3_DEV void run_experts(const StepArgs& a, const ExpertPhase& ph) {
  extern __shared__ __align__(16) unsigned char kk3_dyn_smem[];
  constexpr int S = (MT == 2) ? 8 : 16;
  constexpr int kSlot = MT * kFp4Slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const int npk = a.g.B * a.g.K;
  int nchunks = ld_volatile_int(a.s.chunk_info);
  nchunks = nchunks < 0 ? 0 : (nchunks > npk ? npk : nchunks);
  const long long per_chunk = (long long)ph.tiles * ph.ksteps;
  const long long U = (long long)nchunks * per_chunk;
  if (U == 0) return;
  long long GW = (long long)gridDim.x * kWarps;
  GW = GW < U ? GW : U;
  const long long gw = (long long)blockIdx.x * kWarps + warp;
  if (gw >= GW) return;
  const long long ubeg = U * gw / GW, uend = U * (gw + 1) / GW;
  unsigned char* ring = kk3_dyn_smem + (size_t)warp * kGemvSmemPerWarp;
  float* part_base = a.s.fix_part;
  const int rowbytes = ph.K / 2, sbytes = ph.K / 32;

  auto chunk_expert = [&](int chunk) {
    int e = a.s.chunk_info[1 + chunk * 3];
    return e < 0 ? 0 : (e >= a.g.E ? a.g.E - 1 : e);
  };
  auto at = [&](long long u) {
    ExpertCursor q;
    q.chunk = (int)(u / per_chunk);
    const long long local = u - (long long)q.chunk * per_chunk;
    q.tile = (int)(local / ph.ksteps);
    q.ks = (int)(local % ph.ksteps);
    return q;
  };
  auto step = [&](ExpertCursor& q) {
    if (++q.ks == ph.ksteps) {
      q.ks = 0;
      if (++q.tile == ph.tiles) {
        q.tile = 0;
        ++q.chunk;
      }
    }
  };
  // staging: lane -> (row = lane/2, 16-byte half = lane%2) of every matrix
  const int srow = lane >> 1, shalf = lane & 1;
  auto issue = [&](const ExpertCursor& q, unsigned char* slot) {
    const int e = chunk_expert(q.chunk);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint8_t* src = ph.codes[mt] + (size_t)e * ph.expert_codes + (size_t)(q.tile * 16 + srow) * rowbytes +
                           q.ks * 32 + shalf * 16;
      cp_async16_g(slot + mt * kFp4Slot + srow * kFp4Row + shalf * 16, src);
    }
  };

  ExpertCursor pc = at(ubeg), cc = pc;
  long long pu = ubeg;
#pragma unroll
  for (int i = 0; i < S - 1; ++i) {
    if (pu < uend) {
      issue(pc, ring + (int)((pu - ubeg) % S) * kSlot);
      step(pc);
      ++pu;
    }
    cp_async_commit_g();
  }
  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = 0.0f;
  long long seg_start = ubeg;
  int cur_chunk = -1, expert = 0, first_pair = 0, npairs = 0;
  const __half* xrow = nullptr;
  for (long long u = ubeg; u < uend; ++u) {
    __syncwarp();   // every lane is done with the slot the next issue overwrites
    if (pu < uend) {
      issue(pc, ring + (int)((pu - ubeg) % S) * kSlot);
      step(pc);
      ++pu;
    }
    cp_async_commit_g();
    if (cc.chunk != cur_chunk) {
      cur_chunk = cc.chunk;
      expert = chunk_expert(cur_chunk);
      first_pair = a.s.chunk_info[2 + cur_chunk * 3];
      npairs = a.s.chunk_info[3 + cur_chunk * 3];
      first_pair = first_pair < 0 ? 0 : (first_pair >= npk ? npk - 1 : first_pair);
      npairs = npairs < 0 ? 0 : (npairs > 8 ? 8 : npairs);
      npairs = first_pair + npairs > npk ? npk - first_pair : npairs;
      xrow = nullptr;
      if (r < npairs) {
        const int p = first_pair + r;
        int prow = a.s.pair_row[p];
        prow = prow < 0 ? 0 : (prow >= a.g.B ? a.g.B - 1 : prow);
        xrow = (MT == 2) ? a.s.latent_p + (size_t)prow * a.g.lh : a.s.act_p + (size_t)p * a.g.inter;
      }
    }
    // scales of rows r, r+8 for the unit's two groups, and the activations
    const int rowa = cc.tile * 16 + r;
    unsigned sa[MT], sb[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const uint8_t* sbase = ph.scales[mt] + (size_t)expert * ph.expert_scales + cc.ks * 2;
      sa[mt] = *reinterpret_cast<const unsigned short*>(sbase + (size_t)rowa * sbytes);
      sb[mt] = *reinterpret_cast<const unsigned short*>(sbase + (size_t)(rowa + 8) * sbytes);
    }
    uint4 X[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
    if (xrow) {
      X[0] = ld_act16(xrow + cc.ks * 64 + 8 * c);
      X[1] = ld_act16(xrow + cc.ks * 64 + 32 + 8 * c);
    }
    cp_async_wait_g<S - 1>();
    __syncwarp();
    const unsigned char* slot = ring + (int)((u - ubeg) % S) * kSlot;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        const unsigned wa = lds32(slot + mt * kFp4Slot + r * kFp4Row + g * 16 + 4 * c);
        const unsigned wb = lds32(slot + mt * kFp4Slot + (r + 8) * kFp4Row + g * 16 + 4 * c);
        unsigned ra[4], rb[4];
        e2m1x8_cvt(wa, ra);
        e2m1x8_cvt(wb, rb);
        float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_f16(t, ra[0], rb[0], ra[1], rb[1], X[g].x, X[g].y);
        mma_f16(t, ra[2], rb[2], ra[3], rb[3], X[g].z, X[g].w);
        const float fa = e8m0_to_f32((sa[mt] >> (8 * g)) & 0xffu);
        const float fb = e8m0_to_f32((sb[mt] >> (8 * g)) & 0xffu);
        acc[mt][0] = fmaf(t[0], fa, acc[mt][0]);
        acc[mt][1] = fmaf(t[1], fa, acc[mt][1]);
        acc[mt][2] = fmaf(t[2], fb, acc[mt][2]);
        acc[mt][3] = fmaf(t[3], fb, acc[mt][3]);
      }
    }
    if (cc.ks == ph.ksteps - 1 || u == uend - 1) {
      const long long tile_beg = (long long)cc.chunk * per_chunk + (long long)cc.tile * ph.ksteps;
      const long long first = owner_of(tile_beg, U, GW), lastw = owner_of(tile_beg + ph.ksteps - 1, U, GW);
      bool done = first == lastw;
      if (!done)
        done = stream_k_fixup<MT * 4>(a, part_base, a.s.fix_cnt + cc.chunk * ph.tiles + cc.tile, gw, seg_start == ubeg,
                                      tile_beg, first, lastw, U, GW, *reinterpret_cast<float(*)[MT * 4]>(&acc[0][0]));
      if (done) expert_epilogue<MT>(a, ph, first_pair, npairs, cc.tile, acc);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][i] = 0.0f;
      seg_start = u + 1;
    }
    step(cc);
  }
  cp_async_wait_g<0>();
}

}  // namespace kk3
