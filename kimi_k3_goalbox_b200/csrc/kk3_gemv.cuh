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
  EPI_SITU_GATE,        // single-matrix halves of a situ pair: gate and up tiles are separate jobs of one pass;
  EPI_SITU_UP,          // each publishes its tile, the second to finish a tile forms situ (kimi.py:194-196)
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

constexpr int kMaxJobs = 8;   // jobs of one GEMV pass (the MoE input pass has four)

KK3_DEV long long owner_of(long long u, long long U, long long GW) { return ((u + 1) * GW - 1) / U; }

KK3_DEV void cp_async16_g(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem_dst)),
               "l"(src) : "memory");
}
// streamed weights: L2 evict-first, so the stream does not push code, activations and partials out of L2
KK3_DEV unsigned long long l2_evict_first_policy() {
  unsigned long long pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
KK3_DEV void cp_async16_stream(void* smem_dst, const void* src, unsigned long long pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(
                   (unsigned)__cvta_generic_to_shared(smem_dst)),
               "l"(src), "l"(pol) : "memory");
}
KK3_DEV void cp_async_commit_g() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
KK3_DEV void cp_async_wait_g() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One 64-wide k-step of a 16-row tile: A fragments from this lane's ring slot; activations from the slot
// too when they were staged with it (XS), otherwise from global memory.
template <int NT, int MT, bool XS>
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
      if (XS) {
        X0 = slot[(MT * 4 + nt * 2 + 0) * 32 + lane];
        X1 = slot[(MT * 4 + nt * 2 + 1) * 32 + lane];
      } else {
        const bf16* xr = x + (size_t)n * ldx + ks * 64 + 8 * c;
        X0 = ld_act16(xr);
        X1 = ld_act16(xr + 32);
      }
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

// two floats as a bf16 pair (round to nearest even), lo in the low half (the lower address)
KK3_DEV unsigned pack_bf2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const unsigned*>(&v);
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
// Element index of (source rank, batch row b, channel ch) in a bf16 exchange region (att, shd) of `width`
// channels: [src][width / 16][bp][16]. One 16-row GEMV tile of one source is one contiguous block of bp * 32
// bytes, so the exchange epilogue writes whole 128-byte lines over NVLink; a reader's 8 consecutive channels of
// one row are one 16-byte piece.
KK3_DEV size_t xch_index(const Geo& g, int src, int b, int ch, int width) {
  return (((size_t)src * (width >> 4) + (ch >> 4)) * g.bp + b) * 16 + (ch & 15);
}

// ranks whose regions receive this rank's partial: every rank (peer stores), or only this rank's own region
// when the host reduces the slots with NCCL between launches
KK3_DEV int xdst_lo(const StepArgs& a) { return a.comm_mode == kCommHost ? a.g.rank : 0; }
KK3_DEV int xdst_hi(const StepArgs& a) { return a.comm_mode == kCommHost ? a.g.rank + 1 : a.g.tp; }
// the same for the GEMV epilogues' partials (att, shd): under the push transport they stay local until the
// reading phase pushes them (xch_push)
KK3_DEV int xdst_gemv_lo(const StepArgs& a) { return a.comm_mode == kCommPeer ? 0 : a.g.rank; }
KK3_DEV int xdst_gemv_hi(const StepArgs& a) { return a.comm_mode == kCommPeer ? a.g.tp : a.g.rank + 1; }

// Fused epilogue for one complete 16-row tile. acc[mt][nt][i]: rows row0 + r (+8 for i >= 2), column
// nt*8 + 2c + (i & 1).
// LD: n-tiles whose epilogue loads (the other situ half, the residual operands) are issued together (the warp
// engine keeps it at 2 for its register budget).
template <int NT, int MT, int LD = (NT < 2 ? NT : 2)>
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
  if (j.epi == EPI_SITU_GATE || j.epi == EPI_SITU_UP) {
    // publish this half's bf16-rounded tile (lane-major: each lane's 4*NT values contiguous), then count the
    // halves of the tile; the second half to arrive forms situ(gate, up) from the same lane positions
    const int half = j.epi == EPI_SITU_UP ? 1 : 0;
    float* buf = reinterpret_cast<float*>(const_cast<void*>(j.aux));
    const size_t tile_floats = (size_t)32 * 4 * NT;
    float* mine = buf + ((size_t)half * j.tiles + tile) * tile_floats + (size_t)lane * 4 * NT;
    const float* other = buf + ((size_t)(1 - half) * j.tiles + tile) * tile_floats + (size_t)lane * 4 * NT;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      *reinterpret_cast<float4*>(mine + nt * 4) =
          make_float4(round_bf(acc[0][nt][0]), round_bf(acc[0][nt][1]), round_bf(acc[0][nt][2]), round_bf(acc[0][nt][3]));
    __syncwarp();   // every lane's stores before lane 0's release
    int* cnt = reinterpret_cast<int*>(j.out2) + tile;
    int old = 0;
    if (lane == 0) old = atom_add_acq_rel_gpu(cnt, 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old != 1) return;
    __syncwarp();   // lane 0's acquire before every lane's loads of the other half
    // the other half's loads of two n-tiles at a time before their stores: a load after a store through another
    // pointer cannot be hoisted by the compiler, which made each element one dependent L2 round trip
    constexpr int C = LD;
#pragma unroll
    for (int n0 = 0; n0 < NT; n0 += C) {
      float ov[C][4];
#pragma unroll
      for (int k = 0; k < C; ++k) {
        const float4 t = __ldcg(reinterpret_cast<const float4*>(other + (n0 + k) * 4));   // L2: another SM wrote it
        ov[k][0] = t.x; ov[k][1] = t.y; ov[k][2] = t.z; ov[k][3] = t.w;
      }
#pragma unroll
      for (int k = 0; k < C; ++k) {
        const int nt = n0 + k;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = row0 + r + 8 * (i >> 1);
          const int col = nt * 8 + 2 * c + (i & 1);
          if (row >= j.rows || col >= j.ncols) continue;
          const float mv = round_bf(acc[0][nt][i]);
          const float g = half ? ov[k][i] : mv, u = half ? mv : ov[k][i];
          reinterpret_cast<bf16*>(j.out)[(size_t)col * j.ldo + row] = f2bf(situ_f(g, u));
        }
      }
    }
    if (lane == 0) atomicExch(cnt, 0);
    return;
  }
  if (j.epi == EPI_ROUTED) {
    // prefix[col, row] += bf16(bf16(acc) + shared_red[col, row]) (kimi.py:325-329): all loads first (see the
    // situ pair above), then the stores
    bf16* prefix = reinterpret_cast<bf16*>(j.out);
    const bf16* shared = reinterpret_cast<const bf16*>(j.aux);
    constexpr int C = LD;   // n-tiles whose loads are issued together
#pragma unroll
    for (int n0 = 0; n0 < NT; n0 += C) {
      float pv[C][4], sv[C][4];
#pragma unroll
      for (int k = 0; k < C; ++k)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = row0 + r + 8 * (i >> 1), col = (n0 + k) * 8 + 2 * c + (i & 1);
          const bool ok = row < j.rows && col < j.ncols;
          const size_t o = (size_t)col * j.ldo + row;
          pv[k][i] = ok ? bf2f(prefix[o]) : 0.0f;
          sv[k][i] = ok ? bf2f(shared[o]) : 0.0f;
        }
#pragma unroll
      for (int k = 0; k < C; ++k)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = row0 + r + 8 * (i >> 1), col = (n0 + k) * 8 + 2 * c + (i & 1);
          if (row >= j.rows || col >= j.ncols) continue;
          const float out = round_bf(round_bf(acc[0][n0 + k][i]) + sv[k][i]);
          prefix[(size_t)col * j.ldo + row] = f2bf(pv[k][i] + out);
        }
    }
    return;
  }
  if (j.epi == EPI_EXCHANGE) {
    // bf16(acc) into every rank's region at this rank's slot, layout xch_index (rows = ldo channels, a
    // multiple of 16; padding columns carry the zero products of the zero activation columns). Two shuffles
    // regroup the MMA fragment so that each lane holds 8 contiguous bytes of the n-tile's 256-byte block
    // (column-major, 16 rows per column): one 8-byte store per lane and destination covers the block.
    const int col_l = 2 * c + (r & 1);                     // this lane's column within the n-tile
    const int rw = r >> 1;                                 // row pair R = 2 rw (and R + 8)
    const int woff = col_l * 8 + ((rw & 1) ? 3 + rw : rw); // 4-byte word of the lane's 8-byte piece
    const size_t blk = ((size_t)a.g.rank * (j.ldo >> 4) + tile) * a.g.bp * 16;   // elements
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float* v = acc[0][nt];
      const bool even = (r & 1) == 0;
      // step 1 (partner r ^ 1): even lanes gather column 2c, odd lanes column 2c + 1, rows R, R + 1 (+ 8)
      const float s0 = even ? v[1] : v[0], s1 = even ? v[3] : v[2];
      const float t0 = __shfl_xor_sync(0xffffffffu, s0, 4), t1 = __shfl_xor_sync(0xffffffffu, s1, 4);
      const unsigned w0 = even ? pack_bf2(v[0], t0) : pack_bf2(t0, v[1]);   // rows R, R + 1
      const unsigned w1 = even ? pack_bf2(v[2], t1) : pack_bf2(t1, v[3]);   // rows R + 8, R + 9
      // step 2 (partner rw ^ 1): rw even keeps words (rw, rw + 1), rw odd keeps (rw + 3, rw + 4)
      const unsigned send = (rw & 1) ? w0 : w1;
      const unsigned got = __shfl_xor_sync(0xffffffffu, send, 8);
      const uint2 piece = (rw & 1) ? make_uint2(got, w1) : make_uint2(w0, got);
      const size_t e = blk + (size_t)nt * 128 + (size_t)woff * 2;
      for (int dst = xdst_gemv_lo(a); dst < xdst_gemv_hi(a); ++dst)
        *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(xregion(a, dst, parity) + j.aux_off) + e) = piece;
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
        default:
          break;
      }
    }
  }
}

// Deterministic combination of a tile split over warps first..lastw (see the file comment). `acc` is this
// warp's partial; slot 0/1 of a warp holds its first/other partial tile. Returns true (with the complete
// tile in `acc`) when this warp arrived last and must run the epilogue.
template <int NT, int MT>
KK3_DEV bool stream_k_fixup(const StepArgs& a, float* part_base, int* cnt, long long gw, bool first_seg,
                            long long tile_beg, long long first, long long lastw, long long U, long long GW,
                            float (&acc)[MT][NT][4]) {
  constexpr int NV = MT * NT * 4;
  const int lane = threadIdx.x & 31;
  float* slot = part_base + (size_t)(gw * 2 + (first_seg ? 0 : 1)) * (NV * 32);
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) slot[((mt * NT + nt) * 4 + i) * 32 + lane] = acc[mt][nt][i];
  // one acquire-release RMW publishes this warp's partial (the warp barrier orders every lane's stores before
  // lane 0's release) and, for the last arriver, acquires the others' partials: no separate fences
  __syncwarp();
  int old = 0;
  if (lane == 0) old = atom_add_acq_rel_gpu(cnt, 1);
  old = __shfl_sync(0xffffffffu, old, 0);
  if (old != (int)(lastw - first)) return false;
  __syncwarp();   // lane 0's acquire before every lane's partial loads
  float sum[MT][NT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) sum[mt][nt][i] = 0.0f;
  // plain (non-volatile) L2 loads: the compiler may issue later warps' loads before earlier sums complete
#pragma unroll 8
  for (long long w = first; w <= lastw; ++w) {
    const bool mine = w == gw;
    const long long wbeg = U * w / GW;
    const float* ps = part_base + (size_t)(w * 2 + (wbeg >= tile_beg ? 0 : 1)) * (NV * 32);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          sum[mt][nt][i] += mine ? acc[mt][nt][i] : __ldcg(ps + ((mt * NT + nt) * 4 + i) * 32 + lane);
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][nt][i] = sum[mt][nt][i];
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

constexpr int kGemvSmemPerWarp = 12 * 1024;   // ring bytes per warp (the ring depth follows from the slot size)

// Run a list of dense BF16 jobs with warp-level stream-K over CTAs [cta_lo, cta_hi).
// Producer and consumer walk the warp's unit range with separate cursors; per tile they set up row and
// activation pointers once, per unit they only add the k offset (the per-unit instruction count bounds the
// stream rate at the small batch sizes of decode).
template <int NT, int MT>
KK3_FN void run_gemv(const StepArgs& a, const GemvJob* jobs, int njobs, int cta_lo, int cta_hi, int parity,
                         int bank = 0, int ph = -1) {
  if ((int)blockIdx.x < cta_lo || (int)blockIdx.x >= cta_hi) return;
  extern __shared__ __align__(1024) unsigned char kk3_dyn_smem[];
  constexpr bool XS = NT <= 2;                                   // stage activations with the weights
  constexpr int kSlotVec = (MT * 4 + (XS ? NT * 2 : 0)) * 32;    // uint4 per unit slot
  constexpr int S = kGemvSmemPerWarp / (kSlotVec * 16);          // ring depth in units
  static_assert(S >= 2, "ring too shallow");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;
  const GemvJob& lastj = jobs[njobs - 1];
  const long long U = lastj.ubase + (long long)lastj.tiles * lastj.ksteps;
  long long GW = (long long)(cta_hi - cta_lo) * kWarps;
  GW = GW < U ? GW : U;
  const long long gw = (long long)(blockIdx.x - cta_lo) * kWarps + warp;
  if (U == 0 || gw >= GW) return;
  const long long ubeg = U * gw / GW, uend = U * (gw + 1) / GW;
  const int nunits = (int)(uend - ubeg);
  uint4* ring = reinterpret_cast<uint4*>(kk3_dyn_smem + (size_t)warp * kGemvSmemPerWarp);
  float* part_base = a.s.fix_part + bank * a.g.fix_bank;
  int* cnt_base = a.s.fix_cnt + bank * a.g.cnt_bank;
  const unsigned long long pol = l2_evict_first_policy();
  const bool stamp = ph >= 0 && blockIdx.x == 0 && threadIdx.x == 0;
  // read once: a field of the argument block read inside the loop is reloaded after every asynchronous copy
  // (their asm carries a memory clobber), and the branch on it waits for that load
  const bool trace = a.trace && warp == 0;
  if (stamp) sub_stamp(a, ph, 8);

  // ---- producer: cursor + per-tile pointers
  const Cursor start = locate(jobs, ubeg);
  int p_ji = start.ji, p_tile = start.tile, p_ks = start.ks, p_ksteps = 0, p_tiles = 0;
  const bf16* p_wa[MT];
  const bf16* p_wb[MT];
  const bf16* p_x[NT];
  auto p_setup = [&]() {
    const GemvJob& j = jobs[p_ji];
    p_ksteps = j.ksteps;
    p_tiles = j.tiles;
    int ra = p_tile * 16 + r, rb = ra + 8;
    ra = ra < j.rows ? ra : j.rows - 1;
    rb = rb < j.rows ? rb : j.rows - 1;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const bf16* base = (mt == 0) ? j.w : j.w2;
      p_wa[mt] = base + (size_t)ra * j.K + 8 * c;
      p_wb[mt] = base + (size_t)rb * j.K + 8 * c;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int n = nt * 8 + r;
      p_x[nt] = (XS && n < j.ncols) ? j.x + (size_t)n * j.ldx + 8 * c : nullptr;
    }
  };
  int p_left = nunits, p_slot = 0;
  auto p_issue = [&]() {
    uint4* slot = ring + p_slot * kSlotVec;
    const int off = p_ks * 64;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      cp_async16_stream(slot + (mt * 4 + 0) * 32 + lane, p_wa[mt] + off, pol);
      cp_async16_stream(slot + (mt * 4 + 1) * 32 + lane, p_wa[mt] + off + 32, pol);
      cp_async16_stream(slot + (mt * 4 + 2) * 32 + lane, p_wb[mt] + off, pol);
      cp_async16_stream(slot + (mt * 4 + 3) * 32 + lane, p_wb[mt] + off + 32, pol);
    }
    if (XS) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        if (p_x[nt]) {
          cp_async16_g(slot + (MT * 4 + nt * 2 + 0) * 32 + lane, p_x[nt] + off);
          cp_async16_g(slot + (MT * 4 + nt * 2 + 1) * 32 + lane, p_x[nt] + off + 32);
        }
      }
    }
    p_slot = p_slot + 1 == S ? 0 : p_slot + 1;
    --p_left;
    if (++p_ks == p_ksteps) {
      p_ks = 0;
      if (++p_tile == p_tiles) {
        p_tile = 0;
        ++p_ji;
      }
      if (p_left > 0) p_setup();
    }
  };
  p_setup();
#pragma unroll
  for (int i = 0; i < S - 1; ++i) {
    if (p_left > 0) p_issue();
    cp_async_commit_g();
  }

  // ---- consumer
  int c_ji = start.ji, c_tile = start.tile, c_ks = start.ks, c_slot = 0;
  int c_ksteps = jobs[c_ji].ksteps, c_tiles = jobs[c_ji].tiles;
  const bf16* c_x = jobs[c_ji].x;
  int c_ldx = jobs[c_ji].ldx, c_ncols = jobs[c_ji].ncols;
  float acc[MT][NT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.0f;
  bool first_seg = true;
  for (int n = 0; n < nunits; ++n) {
    if (p_left > 0) p_issue();
    cp_async_commit_g();
    cp_async_wait_g<S - 1>();
    if (stamp && n == 0) sub_stamp(a, ph, 9);
    if (trace && (n & 63) == 0) trace_progress(a, 1, 0x100000 | n);
    mma_step_bf16<NT, MT, XS>(ring + c_slot * kSlotVec, c_x, c_ldx, c_ncols, c_ks, acc);
    c_slot = c_slot + 1 == S ? 0 : c_slot + 1;
    if (c_ks == c_ksteps - 1 || n == nunits - 1) {
      const GemvJob& j = jobs[c_ji];
      const long long tile_beg = j.ubase + (long long)c_tile * c_ksteps;
      const bool inside = tile_beg >= ubeg && tile_beg + c_ksteps <= uend;   // the whole tile is this warp's
      bool done = inside;
      if (!inside) {
        const long long first = owner_of(tile_beg, U, GW), lastw = owner_of(tile_beg + c_ksteps - 1, U, GW);
        done = first == lastw ||
               stream_k_fixup<NT, MT>(a, part_base, cnt_base + j.tile0 + c_tile, gw, first_seg, tile_beg, first,
                                      lastw, U, GW, acc);
      }
      if (done) gemv_epilogue<NT, MT>(a, j, c_tile, acc, parity);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[mt][nt][i] = 0.0f;
      first_seg = false;
    }
    if (++c_ks == c_ksteps) {
      c_ks = 0;
      if (++c_tile == c_tiles) {
        c_tile = 0;
        if (++c_ji < njobs) {
          c_ksteps = jobs[c_ji].ksteps;
          c_tiles = jobs[c_ji].tiles;
          c_x = jobs[c_ji].x;
          c_ldx = jobs[c_ji].ldx;
          c_ncols = jobs[c_ji].ncols;
        }
      }
    }
  }
  cp_async_wait_g<0>();
  warp_end_stamp(a);
  if (stamp) {
    sub_stamp(a, ph, 10);
    sub_stamp(a, ph, 11, (unsigned long long)nunits);
  }
}

// L2 lookahead: weights never depend on activations, so while a latency-bound phase runs, CTAs that are done
// with it prefetch the next GEMV phase's weight matrices into L2 (cp.async.bulk.prefetch). The set is split
// evenly over all CTAs in 64 KB pieces and capped so it fits comfortably in the 126 MB L2.
constexpr long long kPrefetchCap = 96ll << 20;
constexpr unsigned kPrefetchPiece = 64u << 10;

KK3_DEV void prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

KK3_FN void prefetch_jobs(const GemvJob* jobs, int njobs) {
  long long total = 0;
  for (int i = 0; i < njobs; ++i) total += (long long)jobs[i].rows * jobs[i].K * 2 * (jobs[i].w2 ? 2 : 1);
  if (total <= 0 || total > kPrefetchCap) return;
  const long long pieces = (total + kPrefetchPiece - 1) / kPrefetchPiece;
  const long long nthreads = (long long)gridDim.x * 32;
  if (threadIdx.x >= 32) return;
  // lane-major over the CTAs (piece = lane * G + CTA), so every CTA issues pieces / G of them: each bulk
  // prefetch holds the issuing SM's copy engine for a while, and CTA-major pieces made the first few CTAs of
  // the grid (32 pieces each) arrive late at the phase's barrier
  for (long long piece = (long long)threadIdx.x * gridDim.x + blockIdx.x; piece < pieces; piece += nthreads) {
    long long off = piece * kPrefetchPiece;
    for (int i = 0; i < njobs; ++i) {
      for (int m = 0; m < (jobs[i].w2 ? 2 : 1); ++m) {
        const long long bytes = (long long)jobs[i].rows * jobs[i].K * 2;
        if (off < bytes) {
          const long long n = bytes - off < kPrefetchPiece ? bytes - off : kPrefetchPiece;
          prefetch_l2(reinterpret_cast<const unsigned char*>(m ? jobs[i].w2 : jobs[i].w) + off, (unsigned)n);
          i = njobs;
          break;
        }
        off -= bytes;
      }
    }
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

struct ExpertPhase {
  const uint8_t* codes[2];   // gate/up blocks (MT=2) or down blocks (MT=1), expert 0
  const uint8_t* scales[2];
  int rows, K;               // per expert: rows of the matrix, inner dimension
  int tiles, ksteps;
  long long expert_codes;    // bytes of codes per expert (rows * K / 2)
  long long expert_scales;   // bytes of scales per expert (rows * K / 32)
};

// Expert epilogue for one complete tile. `dst[e]` is the output row of this lane's column 2c + e in the chunk
// (null when the chunk has fewer pairs), resolved once per chunk, not per tile. Gate/up (DOWN false, MT == 2):
// rows tile*16 + ..., the FP16 activation row of the pair gets situ(gate, up). Down: the pair's bf16 slot-output
// row; with MT == 2 the tile is two 16-row halves (rows tile*32 + 16 mt + ...), one per "matrix".
template <int MT, bool DOWN>
KK3_DEV void expert_epilogue(int rows, int tile, void* const (&dst)[2], const float (&acc)[MT][1][4]) {
  const int lane = threadIdx.x & 31, r = lane >> 2;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    void* d = dst[i & 1];
    if (d == nullptr) continue;
    if (!DOWN) {
      const int row = tile * 16 + r + 8 * (i >> 1);
      if (row >= rows) continue;
      const float g = round_bf(acc[0][0][i]), u = round_bf(acc[MT - 1][0][i]);
      reinterpret_cast<__half*>(d)[row] = __float2half_rn(round_bf(situ_f(g, u)));
    } else {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int row = tile * 16 * MT + mt * 16 + r + 8 * (i >> 1);
        if (row < rows) reinterpret_cast<bf16*>(d)[row] = f2bf(acc[mt][0][i]);
      }
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


// Stream-K over (expert chunk, tile, k-step) units. Chunks come from the routing step. A unit is a 16-row
// tile x 64 k (two E2M1 groups of 32) of MT matrices; the loop runs over unit pairs (128 k, four groups,
// one 4-byte word of E8M0 scales per row), whose first or last unit may lie outside the warp's range (then
// its groups are skipped). The per-warp cp.async ring carries only weight bytes: 16 rows x 64 code bytes
// per matrix (16-byte chunks XOR-swizzled so that ldmatrix reads are bank-conflict free) and the scale
// word of each row. The FP16 activation rows the CTA's chunks multiply are staged once per phase into a
// shared-memory row cache; rows beyond its capacity are read from L2 through the same generic loads. One
// ldmatrix.x4 gives a lane the four group words of its row; each quad converts them to FP16 in hardware
// (cvt.rn.f16x2.e2m1x2), runs mma.sync per 32-wide group and applies the group scale to the FP32 partial,
// in the same order as a unit at a time.
// E8M0 byte -> 2^(s - 127) from its bits (s << 23), two integer instructions and no table: exact for s in 1..254.
// s = 0 gives 0 instead of the reference's 2^-127 (a weight of at most 6 * 2^-127, below the resolution of any
// FP32 sum it enters); s = 255 gives inf instead of the reference's NaN group (the output is not finite either way).
KK3_DEV float e8m0_bits(unsigned s) { return __uint_as_float(s << 23); }

constexpr int kExpRing = 10240;           // per-warp ring bytes: four MT=2 pair slots (2560 B) or six MT=1
constexpr int kExpXCache = 56 * 1024;     // per-CTA activation row cache, after the rings
constexpr int kExpSmem = kWarps * kExpRing + kExpXCache;

KK3_DEV void ldsm4(unsigned (&r)[4], unsigned addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
KK3_DEV unsigned lds32_u(unsigned addr) {
  unsigned v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
// f16 MMA without `volatile`, so the compiler may interleave independent groups
KK3_DEV void mma_f16_nv(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0, unsigned b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

KK3_DEV void cp_async4_ca(void* smem_dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((unsigned)__cvta_generic_to_shared(smem_dst)),
               "l"(src) : "memory");
}

KK3_DEV uint4 ld_cg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// MT matrices per unit: gate and up (DOWN false), or the down projection as one matrix (MT == 1) or as two
// adjacent 16-row tiles streamed together (MT == 2, "row pairs": codes[1] / scales[1] point 16 rows further,
// tiles count 32-row pairs), which shares each activation load and each unit's fixed costs between two tiles.
template <int MT, bool DOWN = (MT == 1)>
KK3_FN void run_experts(const StepArgs& a, const ExpertPhase& ph) {
  extern __shared__ __align__(1024) unsigned char kk3_dyn_smem[];
  __shared__ unsigned long long s_mask;    // gate/up: batch rows staged (bit b = latent row b)
  __shared__ int s_first, s_count;        // down: pairs [s_first, s_first + s_count) staged
  __shared__ int s_rowmap[kMaxBatch];     // gate/up: cache slot i holds latent row s_rowmap[i]
  constexpr int kCode = 16 * 64;                  // code bytes per matrix and unit pair
  // scale bytes per matrix and unit pair: the 16-byte window (four pairs) of every row, or, when a row's scales
  // are not a multiple of 16 bytes, the tile's whole scale block (16 rows x K/32 bytes, contiguous)
  constexpr int kScale = MT == 2 ? 256 : 512;
  constexpr int kTileRows = DOWN ? 16 * MT : 16;   // weight rows a tile index advances by
  constexpr int kSlot = MT * (kCode + kScale);
  constexpr int S = (kExpRing / kSlot) > 12 ? 12 : (kExpRing / kSlot);
  static_assert(S >= 4, "ring too shallow");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, r = lane >> 2, c = lane & 3;

  // values of the unit loop live in registers; values used only when a tile or chunk changes are re-read
  // from the descriptor there (once per ksteps units)
  const int tiles = ph.tiles, ksteps = ph.ksteps;
  const int npk = a.g.B * a.g.K;
  const bool trace = a.trace != 0;
  int nchunks = __ldcg(a.s.chunk_info);
  nchunks = nchunks < 0 ? 0 : (nchunks > npk ? npk : nchunks);
  const int per_chunk = tiles * ksteps;      // <= 512 tiles x 128 k-steps
  const int U = nchunks * per_chunk;         // <= 2048 chunks: fits 32 bits; even (ksteps is even)
  if (U == 0) return;                        // the same for every thread of the grid
  // warps get whole unit pairs: warp w owns pairs [UP * w / GW, UP * (w + 1) / GW), so no pair is split
  // between warps and the unit loop has no partial pairs
  const int UP = U >> 1;
  int GW = gridDim.x * kWarps;
  GW = GW < UP ? GW : UP;

  // routing-table values are clamped so that a routing fault can never address outside the buffers
  auto chunk_expert = [&](int chunk) {
    const int e = __ldcg(a.s.chunk_info + 1 + chunk * 3);
    return e < 0 ? 0 : (e >= a.g.E ? a.g.E - 1 : e);
  };
  auto chunk_pairs = [&](int chunk, int& fp, int& np) {
    fp = __ldcg(a.s.chunk_info + 2 + chunk * 3);
    np = __ldcg(a.s.chunk_info + 3 + chunk * 3);
    fp = fp < 0 ? 0 : (fp >= npk ? npk - 1 : fp);
    np = np < 0 ? 0 : (np > 8 ? 8 : np);
    np = fp + np > npk ? npk - fp : np;
  };
  auto pair_batch_row = [&](int p) {
    const int b = __ldcg(a.s.pair_row + p);
    return b < 0 ? 0 : (b >= a.g.B ? a.g.B - 1 : b);
  };

  // ---- stage the activation rows of this CTA's chunks (all threads, before any warp leaves)
  const int xrow_bytes = ph.K * 2, xstride = xrow_bytes + 64;   // +64 B: rows alternate bank halves
  const int cap = kExpXCache / xstride;
  unsigned char* xcache = kk3_dyn_smem + kWarps * kExpRing;
  const int cw0 = blockIdx.x * kWarps;
  if (threadIdx.x == 0) {
    unsigned long long mask = 0ull;
    int first = 0, count = 0;
    if (cw0 < GW) {
      const int cbeg = 2 * (int)((long long)UP * cw0 / GW);
      const int cend = 2 * (int)((long long)UP * (cw0 + kWarps < GW ? cw0 + kWarps : GW) / GW);
      int fp_lo, np_lo, fp_hi, np_hi;
      chunk_pairs(cbeg / per_chunk, fp_lo, np_lo);
      chunk_pairs((cend - 1) / per_chunk, fp_hi, np_hi);
      const int p_lo = fp_lo, p_hi = fp_hi + np_hi > p_lo ? fp_hi + np_hi : p_lo;
      if (!DOWN) {
        for (int p = p_lo; p < p_hi; ++p) mask |= 1ull << pair_batch_row(p);
        int n = 0;
        for (int b = 0; b < a.g.B; ++b) {
          if (!((mask >> b) & 1ull)) continue;
          if (n == cap) {
            mask &= ~(1ull << b);   // beyond capacity: read from L2
            continue;
          }
          s_rowmap[n++] = b;
        }
        count = n;
      } else {
        first = p_lo;
        count = p_hi - p_lo < cap ? p_hi - p_lo : cap;
      }
    }
    s_mask = mask;
    s_first = first;
    s_count = count;
  }
  __syncthreads();
  {
    const int pieces_per_row = xrow_bytes / 16;
    const int total = s_count * pieces_per_row;
    for (int q = threadIdx.x; q < total; q += kThreads) {
      const int i = q / pieces_per_row, col = q - i * pieces_per_row;
      const __half* src = !DOWN ? a.s.latent_p + (size_t)s_rowmap[i] * a.g.lh
                                    : a.s.act_p + (size_t)(s_first + i) * a.g.inter;
      cp_async16_g(xcache + i * xstride + col * 16, src + col * 8);
    }
    cp_async_commit_g();
    cp_async_wait_g<0>();
    __syncthreads();
  }
  const unsigned long long xmask = s_mask;
  const int xfirst = s_first, xcount = s_count;
  if (blockIdx.x == 0 && threadIdx.x == 0) sub_stamp(a, kk3_cur_phase, 1);   // activation rows staged

  const int gw = cw0 + warp;
  if (gw >= GW) return;
  const int ubeg = 2 * (int)((long long)UP * gw / GW), uend = 2 * (int)((long long)UP * (gw + 1) / GW);
  unsigned char* ring = kk3_dyn_smem + (size_t)warp * kExpRing;
  if (trace) trace_warp(a, 1);

  // ---- unit pairs: pair P holds units 2P, 2P + 1 (ksteps is even, so a pair never spans two tiles)
  const int kpairs = ksteps >> 1;
  const int pbeg = ubeg >> 1, npairs = ((uend + 1) >> 1) - pbeg;
  const int c0 = (2 * pbeg) / per_chunk;
  const int rem0 = 2 * pbeg - c0 * per_chunk;
  const int t0 = rem0 / ksteps, kp0 = (rem0 - t0 * ksteps) >> 1;

  // ---- producer (weights into the ring, S - 1 pairs ahead); per-lane slot offsets are fixed
  const unsigned ring_s = (unsigned)__cvta_generic_to_shared(ring);
  int p_chunk = c0, p_tile = t0, p_kp = kp0;
  const int prow = lane >> 2, pq = lane & 3;                                   // row (and row + 8), 16-byte chunk
  const unsigned p_dst_code = prow * 64 + ((pq ^ ((prow >> 1) & 3)) << 4);     // swizzled chunk of the row
  const uint8_t* p_code[MT];   // this lane's 16 code bytes of row prow of the current pair, per matrix
  const size_t rowbytes = (size_t)(ph.K >> 1), sbytes = (size_t)(ph.K >> 5);
  // scales with 16-byte copies (L1 bypassed): windowed (K % 512 == 0) - lane (mt, row) copies the 16-byte
  // window of its row holding pairs 4w..4w+3 - or whole-tile (K <= 512, or K <= 1024 for MT = 1) - lane
  // (mt, piece) copies one 16-byte piece of the tile's contiguous 16 x K/32-byte scale block
  const bool swin = (sbytes & 15) == 0;
  const int spm = MT == 2 ? 16 : 32;                                             // lanes per matrix
  const int scl_mt = lane / spm, scl_i = lane % spm;                             // matrix, row or piece
  const bool scl_lane = scl_mt < MT && (swin ? scl_i < 16 : scl_i < (int)sbytes);
  const unsigned p_dst_scl = MT * kCode + scl_mt * kScale + scl_i * 16;
  const uint8_t* p_scl = ph.scales[0];   // this lane's window row (plus 16 * window) or tile piece
  const unsigned long long pol = l2_evict_first_policy();   // codes are read once per step
  int p_echunk = -1;   // chunk whose expert id is cached in p_e (tiles of a chunk share the expert)
  size_t p_e = 0;
  auto p_setup = [&]() {
    if (p_chunk != p_echunk) {
      p_e = (size_t)chunk_expert(p_chunk);
      p_echunk = p_chunk;
    }
    const size_t e = p_e;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
      p_code[mt] = ph.codes[mt] + e * ph.expert_codes + (size_t)(p_tile * kTileRows + prow) * rowbytes + p_kp * 64 + pq * 16;
    if (scl_lane)
      p_scl = ph.scales[scl_mt] + e * ph.expert_scales +
              (swin ? (size_t)(p_tile * kTileRows + scl_i) * sbytes : (size_t)p_tile * kTileRows * sbytes + scl_i * 16);
  };
  // A scale window (the scales of 4 pairs, or of the whole tile) is copied once, with the first of its pairs the
  // warp issues, into the scale area of window slot (window count % S); the consumer counts windows the same way.
  // Window slot w is reused S windows later, when the consumer has left window w behind (every window holds at
  // least one pair and the producer runs S - 1 pairs ahead).
  const int wmask = swin ? 3 : 0x7fffffff;   // (kp & wmask) == 0: kp opens a window
  int p_left = npairs, p_slot = 0, p_wslot = S - 1;
  bool p_first = true;
  auto p_issue = [&]() {
    const unsigned slot = ring_s + p_slot * kSlot;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;"
                   ::"r"(slot + mt * kCode + p_dst_code), "l"(p_code[mt]), "l"(pol) : "memory");
      asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;"
                   ::"r"(slot + mt * kCode + 512 + p_dst_code), "l"(p_code[mt] + 8 * rowbytes), "l"(pol) : "memory");
      p_code[mt] += 64;
    }
    if (p_first || (p_kp & wmask) == 0) {
      p_wslot = p_wslot + 1 == S ? 0 : p_wslot + 1;
      if (scl_lane)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ring_s + p_wslot * kSlot + p_dst_scl),
                     "l"(p_scl + (swin ? (p_kp >> 2) * 16 : 0)) : "memory");
    }
    p_first = false;
    p_slot = p_slot + 1 == S ? 0 : p_slot + 1;
    --p_left;
    if (++p_kp == kpairs) {
      p_kp = 0;
      if (++p_tile == tiles) {
        p_tile = 0;
        ++p_chunk;
      }
      if (p_left > 0) p_setup();
    }
  };
  p_setup();
#pragma unroll 1
  for (int i = 0; i < S - 1; ++i) {
    if (p_left > 0) p_issue();
    cp_async_commit_g();
  }
  if (trace) trace_warp(a, 4);

  // ---- activations of the current chunk for this lane's pair r (generic pointer: a cached row in shared
  // memory or an L2 row); lanes without a pair read any cached row, their MMA columns are never stored
  int c_chunk = c0, c_tile = t0, c_kp = kp0;
  int c_fp = 0, c_np = 0;
  // lanes without a pair read a cached row (or a real global row when nothing fits the cache)
  const unsigned char* xdead = cap > 0 ? xcache
                                       : reinterpret_cast<const unsigned char*>(!DOWN ? a.s.latent_p : a.s.act_p);
  const unsigned char* xp = xdead;
  int x_off = 0;             // byte offset of this lane's row in the cache (when cached)
  bool x_shared = cap > 0;   // every lane's row of the current chunk is in the cache (shared-memory loads)
  void* out_row[2] = {nullptr, nullptr};   // epilogue targets of this lane's columns 2c, 2c + 1
  auto x_setup = [&]() {
    chunk_pairs(c_chunk, c_fp, c_np);
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = 2 * c + e;
      out_row[e] = nullptr;
      if (col >= c_np) continue;
      const int pc = c_fp + col;
      if (!DOWN) {
        out_row[e] = a.s.act_p + (size_t)pc * a.g.inter;
      } else {
        int slot = __ldcg(a.s.pair_slot + pc);
        slot = slot < 0 ? 0 : (slot >= a.g.K ? a.g.K - 1 : slot);
        out_row[e] = a.s.out_slot + ((size_t)pair_batch_row(pc) * a.g.K + slot) * a.g.lh;
      }
    }
    xp = xdead;
    x_off = 0;
    bool cached = cap > 0;
    if (r < c_np) {
      const int p = c_fp + r;
      if (!DOWN) {
        const int b = pair_batch_row(p);
        cached = (xmask >> b) & 1ull;
        x_off = cached ? __popcll(xmask & ((1ull << b) - 1ull)) * xstride : 0;
        xp = cached ? xcache + x_off : reinterpret_cast<const unsigned char*>(a.s.latent_p + (size_t)b * a.g.lh);
      } else {
        const int i = p - xfirst;
        cached = i >= 0 && i < xcount;
        x_off = cached ? i * xstride : 0;
        xp = cached ? xcache + x_off : reinterpret_cast<const unsigned char*>(a.s.act_p + (size_t)p * a.g.inter);
      }
    }
    x_shared = __all_sync(0xffffffffu, cached);
  };
  x_setup();

  // ---- consumer; per-lane read offsets inside a slot are fixed
  int c_slot = 0;
  const int lrow = lane & 7, lq = lane >> 3;   // ldmatrix: this lane addresses row lrow (+8) of chunk lq
  const unsigned c_ldsm = lrow * 64 + ((lq ^ ((lrow >> 1) & 3)) << 4);
  // this lane's scale words (rows r, r + 8) of pair kp: + (kp & 3) * 4 (windowed) or + kp * 4 (whole tile)
  const unsigned c_scl_a = MT * kCode + r * (swin ? 16u : (unsigned)sbytes);
  const unsigned c_scl_b = MT * kCode + (r + 8) * (swin ? 16u : (unsigned)sbytes);
  const int c_kmask = swin ? 3 : 0x7fffffff;
  float acc[MT][1][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][0][i] = 0.0f;
  int c_wslot = S - 1;   // window slot of the current pair's scales (counted as the producer counts)
  for (int n = 0; n < npairs; ++n) {
    __syncwarp();   // every lane is done with the slot the next issue overwrites
    if (p_left > 0) p_issue();
    cp_async_commit_g();
    cp_async_wait_g<S - 1>();
    __syncwarp();
    if (trace && n < 2) trace_warp(a, 5 | (n << 8));
    const unsigned slot = ring_s + c_slot * kSlot;
    c_slot = c_slot + 1 == S ? 0 : c_slot + 1;
    // this pair's activation pieces: k = 128 kp + 64 u + 32 g + 8c, group j = 2u + g; each next one is
    // loaded while the previous group is being multiplied
    const int xko = c_kp * 256 + c * 16;
    auto ldx = [&](int j) -> uint4 {
      if (x_shared) return *reinterpret_cast<const uint4*>(xcache + x_off + xko + j * 64);   // shared
      return *reinterpret_cast<const uint4*>(xp + xko + j * 64);                              // generic
    };
    uint4 xn = ldx(0);
    if (n == 0 || (c_kp & wmask) == 0) c_wslot = c_wslot + 1 == S ? 0 : c_wslot + 1;
    unsigned wa[MT][4], wb[MT][4], sa[MT], sb[MT];   // group words and scale words of rows r and r + 8
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      ldsm4(wa[mt], slot + mt * kCode + c_ldsm);
      ldsm4(wb[mt], slot + mt * kCode + 512 + c_ldsm);
      const unsigned char* sl = ring + (size_t)c_wslot * kSlot + mt * kScale + (c_kp & c_kmask) * 4;
      sa[mt] = *reinterpret_cast<const unsigned*>(sl + c_scl_a);
      sb[mt] = *reinterpret_cast<const unsigned*>(sl + c_scl_b);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 X = xn;
      if (j < 3) xn = ldx(j + 1);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        unsigned ra[4], rb[4];
        e2m1x8_cvt(wa[mt][j], ra);
        e2m1x8_cvt(wb[mt][j], rb);
        float t[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_f16_nv(t, ra[0], rb[0], ra[1], rb[1], X.x, X.y);
        mma_f16_nv(t, ra[2], rb[2], ra[3], rb[3], X.z, X.w);
        // 2^(s - 127) from the scale byte's bits (see e8m0_bits)
        const float fa = e8m0_bits((sa[mt] >> (8 * j)) & 0xffu), fb = e8m0_bits((sb[mt] >> (8 * j)) & 0xffu);
        acc[mt][0][0] = fmaf(t[0], fa, acc[mt][0][0]);
        acc[mt][0][1] = fmaf(t[1], fa, acc[mt][0][1]);
        acc[mt][0][2] = fmaf(t[2], fb, acc[mt][0][2]);
        acc[mt][0][3] = fmaf(t[3], fb, acc[mt][0][3]);
      }
    }
    if (c_kp == kpairs - 1 || n == npairs - 1) {
      const int tile_beg = c_chunk * per_chunk + c_tile * ksteps;
      // the whole tile is this warp's: no fix-up (owners are computed only for split tiles, a 64-bit division);
      // ownership is by unit pairs, so the fix-up works in pairs
      bool done = tile_beg >= ubeg && tile_beg + ksteps <= uend;
      if (!done) {
        const int pt = tile_beg >> 1;
        const long long first = owner_of(pt, UP, GW), lastw = owner_of(pt + kpairs - 1, UP, GW);
        done = first == lastw ||
               stream_k_fixup<1, MT>(a, a.s.fix_part, a.s.fix_cnt + c_chunk * tiles + c_tile, gw, tile_beg <= ubeg,
                                     pt, first, lastw, UP, GW, acc);
      }
      if (done) expert_epilogue<MT, DOWN>(ph.rows, c_tile, out_row, acc);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][0][i] = 0.0f;
    }
    if (++c_kp == kpairs) {
      c_kp = 0;
      if (++c_tile == tiles) {
        c_tile = 0;
        ++c_chunk;
        if (n + 1 < npairs) x_setup();
      }
    }
  }
  cp_async_wait_g<0>();
  warp_end_stamp(a);
  if (trace) trace_warp(a, 11);
}

}  // namespace kk3
