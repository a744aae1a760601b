// kk3_tc_gemv.cuh - the BF16 projections of the decode step on the 5th-generation tensor cores
// (tcgen05.mma kind::f16, sm_100a), for the batch classes of 17-64 rows (NT = 4 and 8).
//
// At those batches the warp-level mma.sync engine (run_gemv, kk3_gemv.cuh) is bound by its activation traffic:
// every 16-row weight tile re-reads the whole activation k-step (NT * 8 rows) from L2 and issues NT times
// the MMAs of a batch-8 step. Here one MMA covers a 128-row weight block and the whole batch
// (y[b, n] = sum_k x[b, k] W[n, k] with the weights as M = 128 and the batch as N = 8 NT), the activations of
// a k-step are staged once per CTA, and the FP32 accumulator stays in TMEM for the unit.
//
// Work split: CTA-level stream-K over the pass's (job, 128-row block, k-step) space, an equal contiguous range per
// CTA (see run_gemv_tc). Per k-step of 64:
//  - all 512 threads copy the stage with 16-byte cp.async: 128 weight rows x 128 bytes (L2 evict-first) and N
//    activation rows x 128 bytes (zeros past the batch), into the 128-byte-swizzled K-major layout
//    (8-row atoms of 1024 bytes, 16-byte chunk j of row r at r * 128 + ((j ^ (r & 7)) << 4));
//  - each thread waits for its own copies, makes them visible to the async proxy (fence.proxy.async: the
//    copies are generic-proxy writes and the tensor core reads through the async proxy), then the CTA
//    synchronises and thread 0 issues four K = 16 MMAs and commits them to the stage's mbarrier;
//  - a stage is refilled only after the mbarrier of the MMAs that read it completed, two k-steps later, so
//    the MMA latency stays off the copy path; the copies run S - 2 k-steps ahead of the MMAs, across blocks
//    (a k-step streams in ~1 us while its four MMAs finish in well under that).
// At the end of a segment (the CTA's k-steps of one block) warps 0-3 read the accumulator (TMEM lane = block
// row) with tcgen05.ld. A block done by one CTA goes straight to the epilogue; otherwise each contributor
// writes its FP32 partial to the stream-K bank and the last to arrive sums them in CTA order (deterministic)
// before the epilogue. The 128 x N block is staged column-major in shared memory. Plain stores (bf16, FP32 sigmoid, latent) go out
// column by column in 16-byte pieces; every other epilogue is the GEMV engine's gemv_epilogue, run by eight
// warps on one 16-row tile each in the mma.sync fragment layout, so the fused epilogues (exchange stores,
// situ pairs, logits keys, residual update) are shared with the mma.sync path. The reduction and the epilogue
// are separate (not inlined) functions, so their registers do not spill in the streaming loop.
#pragma once
#include "kk3_tcgen05.cuh"

namespace kk3 {

constexpr int kTcgRows = 128;                 // M: weight rows per block
constexpr int kTcgStageA = kTcgRows * 128;    // bytes of one weight stage (128 rows x 64 bf16)

template <int NT>
struct TcGemvShape {
  static constexpr int N = NT * 8;                               // batch columns of the MMA
  static constexpr int kStageB = N * 128;                        // bytes of one activation stage
  static constexpr int kStage = kTcgStageA + kStageB;            // a multiple of 1024: stages stay swizzle-aligned
  static constexpr int kStagingStride = kTcgRows + 4;            // floats per staged result column (column-major)
  static constexpr int kStaging = N * kStagingStride * 4;
  static constexpr int kCtl = 1024;                              // mbarriers, TMEM address, pass plan
  static constexpr int kStagesFit = (kExpSmem - kStaging - kCtl) / kStage;   // within the step's dynamic smem
  static constexpr int S = kStagesFit > 8 ? 8 : kStagesFit;
  static constexpr int kTmemCols = N < 32 ? 32 : N;              // power of two >= 32
  static_assert(kStage % 1024 == 0, "stages must keep the 1024-byte swizzle atoms aligned");
  static constexpr int kBytes = S * kStage + kStaging + kCtl;
  static_assert(S >= 3, "too few stages");
  static_assert(kBytes <= kExpSmem, "the step kernel's dynamic shared memory is sized by the expert engine");
};

// Instruction descriptor, kind::f16: D = F32, A = B = BF16, both K-major, M = 128, N.
KK3_DEV unsigned idesc_bf16_f32(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(n >> 3) << 17) | ((unsigned)(kTcgRows >> 4) << 24);
}
KK3_DEV void umma_bf16(unsigned d, unsigned long long adesc, unsigned long long bdesc, unsigned idesc,
                       unsigned accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// 32 TMEM lanes (one per thread of the warp) x 16 consecutive 32-bit columns
KK3_DEV void tmem_ld16(unsigned taddr, float (&v)[16]) {
  unsigned r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr) : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
KK3_DEV void st_shared_zero16(unsigned addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
}

// Pass plan (thread 0 writes it into shared memory): per job its 128-row blocks, k-steps and first k-step in
// the pass's k-step space (job-major, then block, then k-step).
struct TcPlan {
  int njobs;
  long long total;                   // k-steps of the pass
  long long ubase[kMaxJobs + 1];
  int blocks[kMaxJobs];
  int ksteps[kMaxJobs];
  int bbase[kMaxJobs];               // first block (counter index) of each job
};

KK3_DEV void tc_plan(const GemvJob* jobs, int njobs, TcPlan& p) {
  long long u = 0;
  int b = 0;
  for (int i = 0; i < njobs; ++i) {
    p.blocks[i] = (jobs[i].rows + kTcgRows - 1) / kTcgRows;
    p.ksteps[i] = jobs[i].K / 64;
    p.ubase[i] = u;
    p.bbase[i] = b;
    u += (long long)p.blocks[i] * p.ksteps[i];
    b += p.blocks[i];
  }
  p.ubase[njobs] = u;
  p.njobs = njobs;
  p.total = u;
}

// (job, block, k-step) of position u of the k-step space
struct TcPos {
  int job, block, ks;
};
KK3_DEV TcPos tc_locate(const TcPlan& p, long long u) {
  int j = 0;
  while (j + 1 < p.njobs && u >= p.ubase[j + 1]) ++j;
  const long long r = u - p.ubase[j];
  TcPos t;
  t.job = j;
  t.block = (int)(r / p.ksteps[j]);
  t.ks = (int)(r - (long long)t.block * p.ksteps[j]);
  return t;
}

constexpr int kTcgLag = 2;   // a stage is refilled once the MMAs of 2 k-steps ago completed

// Profiling contexts only (warp_ts allocated): CTA-level event k of this pass into the per-warp stamp slot k of
// the CTA (0 start, 1 first k-step's data landed, 2 last k-step's MMAs issued, 3 last segment's MMAs done,
// 4 its partial published or staged, 5 after its reduction, 6 after its epilogue, 7 pass end).
KK3_DEV void tc_stamp(const StepArgs& a, int k) {
  if (a.s.warp_ts && threadIdx.x == 0) {
    const int ph = kk3_cur_phase;
    if (ph >= 0 && ph < kArrivePhases) a.s.warp_ts[((size_t)ph * gridDim.x + blockIdx.x) * kWarps + k] = globaltimer();
  }
}

// Sum of a split block's partials into the staging block (all threads; CTA order, deterministic). Not inlined, so
// that its registers (all loads of four contributors in flight per thread) never spill in the streaming loop.
template <int NT>
KK3_FN void tc_reduce_block(const float* part_base, float* staging, long long first, long long lastc,
                            long long bstart, long long U, long long G) {
  constexpr int N = NT * 8, E = kTcgRows * N / 4 / kThreads;   // float4 elements per thread
  static_assert(E * kThreads == kTcgRows * N / 4, "reduction elements per thread");
  const int ncon = (int)(lastc - first) + 1;
  float4 acc[E];
#pragma unroll
  for (int k = 0; k < E; ++k) acc[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (int k0 = 0; k0 < ncon; k0 += 4) {
    float4 v[4][E];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const long long c = first + k0 + t;
      const float4* src = reinterpret_cast<const float4*>(
          part_base + ((size_t)c * 2 + ((U * c / G >= bstart) ? 0 : 1)) * kTcgRows * N);
#pragma unroll
      for (int k = 0; k < E; ++k)
        v[t][k] = k0 + t < ncon ? __ldcg(src + threadIdx.x + k * kThreads) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
      for (int k = 0; k < E; ++k) {
        acc[k].x += v[t][k].x; acc[k].y += v[t][k].y; acc[k].z += v[t][k].z; acc[k].w += v[t][k].w;
      }
  }
#pragma unroll
  for (int k = 0; k < E; ++k) {
    const int e = threadIdx.x + k * kThreads, q = e / kTcgRows, row = e - q * kTcgRows;   // partial: [N/4][128]
    float* col = staging + (4 * q) * TcGemvShape<NT>::kStagingStride + row;   // staging: [N][128 + 4]
    col[0] = acc[k].x;
    col[TcGemvShape<NT>::kStagingStride] = acc[k].y;
    col[2 * TcGemvShape<NT>::kStagingStride] = acc[k].z;
    col[3 * TcGemvShape<NT>::kStagingStride] = acc[k].w;
  }
}

// Epilogue of one finished 128 x N block from the staging buffer (all threads). Each kind of epilogue has its own
// compact loop over 8-row pieces of one output column (16-byte stores where the row stride allows): the block
// is finished once per pass by whichever CTA completes it, so its code runs cold from the instruction cache,
// and the GEMV engine's per-tile gemv_epilogue (every kind, fully unrolled for the fragment layout) took up to
// ~25 us there. The arithmetic and rounding are the same as gemv_epilogue's (kimi.py:304, :308, :317, :325-331,
// :343-347). sflags: 8 ints of shared memory for the situ pairing. Not inlined, like tc_reduce_block.
template <int NT>
KK3_FN void tc_epilogue_block(const StepArgs& a, const GemvJob& j, int block, const float* staging, int parity,
                              volatile int* sflags) {
  constexpr int N = NT * 8, SS = TcGemvShape<NT>::kStagingStride;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = block * kTcgRows;
  const int nrows = j.rows - row0 < kTcgRows ? j.rows - row0 : kTcgRows;
  const bool vec = (j.ldo & 7) == 0;   // 8-row pieces are 16-byte aligned in the output
  const int epi = j.epi;
  if (epi == EPI_SITU_GATE || epi == EPI_SITU_UP) {
    // publish this half's bf16-rounded tiles ([N][16] floats per 16-row tile), count the halves of each tile;
    // the second half to arrive forms situ(gate, up) (kimi.py:194-196)
    const int half = epi == EPI_SITU_UP ? 1 : 0;
    const int ntiles = (nrows + 15) >> 4;
    float* buf = reinterpret_cast<float*>(const_cast<void*>(j.aux));
    const size_t tf = (size_t)16 * N;
    #pragma unroll 1
    for (int e = tid; e < ntiles * N * 4; e += kThreads) {   // float4 of rows 4q .. 4q + 3 of column n, tile t
      const int t = e / (N * 4), rem = e - t * N * 4, n = rem >> 2, q = rem & 3;
      const float4 v = *reinterpret_cast<const float4*>(staging + n * SS + t * 16 + q * 4);
      *reinterpret_cast<float4*>(buf + ((size_t)half * j.tiles + block * 8 + t) * tf + n * 16 + q * 4) =
          make_float4(round_bf(v.x), round_bf(v.y), round_bf(v.z), round_bf(v.w));
    }
    __syncthreads();
    int* cnt = reinterpret_cast<int*>(j.out2) + block * 8;
    if (tid < ntiles) {
      __threadfence();
      sflags[tid] = atom_add_acq_rel_gpu(cnt + tid, 1) == 1;
    }
    __syncthreads();
    __threadfence();
    #pragma unroll 1
    for (int p = tid; p < ntiles * N * 2; p += kThreads) {   // 8-row piece h of column n, tile t
      const int t = p / (N * 2), rem = p - t * N * 2, n = rem >> 1, h = rem & 1;
      if (!sflags[t] || n >= j.ncols) continue;
      const int rr = t * 16 + h * 8;
      const float* oth = buf + ((size_t)(1 - half) * j.tiles + block * 8 + t) * tf + n * 16 + h * 8;
      const float4 o0 = __ldcg(reinterpret_cast<const float4*>(oth)), o1 = __ldcg(reinterpret_cast<const float4*>(oth + 4));
      const float ov[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
      float res[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float mv = round_bf(staging[n * SS + rr + e]);
        res[e] = situ_f(half ? ov[e] : mv, half ? mv : ov[e]);
      }
      bf16* out = reinterpret_cast<bf16*>(j.out) + (size_t)n * j.ldo + row0 + rr;
      if (vec && rr + 8 <= nrows) {
        *reinterpret_cast<uint4*>(out) = pack8(res);
      } else {
        for (int e = 0; e < 8 && rr + e < nrows; ++e) out[e] = f2bf(res[e]);
      }
    }
    __syncthreads();
    if (tid < ntiles && sflags[tid]) atomicExch(cnt + tid, 0);
    __syncthreads();
    return;
  }
  if (epi == EPI_LOGITS) {
    // argmax keys: warp w takes columns w, w + 16, ...; per column the largest (value, lowest index) key of the
    // block's rows, one atomicMax per column (kimi.py:218-227, :331)
    #pragma unroll 1
    for (int n = warp; n < N; n += kWarps) {
      unsigned long long best = 0ull;
      #pragma unroll 1
      for (int r = lane; r < nrows; r += 32) {
        const unsigned long long k = argmax_key(round_bf(staging[n * SS + r]), (unsigned)(row0 + r + j.aux_off));
        best = k > best ? k : best;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
      }
      if (lane == 0 && n < j.ncols && best != 0ull)
        atomicMax(reinterpret_cast<unsigned long long*>(const_cast<void*>(j.aux)) + n, best);
    }
  }
  #pragma unroll 1
  for (int p = tid; p < N * 16; p += kThreads) {   // 8-row piece of column n
    const int n = p >> 4, rr = (p & 15) * 8;
    if (rr >= nrows || (n >= j.ncols && epi != EPI_EXCHANGE)) continue;
    float v[8];
    const float4 s0 = *reinterpret_cast<const float4*>(staging + n * SS + rr);
    const float4 s1 = *reinterpret_cast<const float4*>(staging + n * SS + rr + 4);
    v[0] = s0.x; v[1] = s0.y; v[2] = s0.z; v[3] = s0.w; v[4] = s1.x; v[5] = s1.y; v[6] = s1.z; v[7] = s1.w;
    const size_t o = (size_t)n * j.ldo + row0 + rr;
    const bool full = vec && rr + 8 <= nrows;
    if (epi == EPI_EXCHANGE) {
      // this rank's slot of every destination's region (xch_index layout; rows = ldo channels, a multiple of
      // 16); padding columns carry the zero products of the zero activation columns
      const uint4 b = pack8(v);
      const size_t e = xch_index(a.g, a.g.rank, n, row0 + rr, j.ldo);
      for (int dst = xdst_gemv_lo(a); dst < xdst_gemv_hi(a); ++dst)
        *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(xregion(a, dst, parity) + j.aux_off) + e) = b;
    } else if (epi == EPI_ROUTED) {
      // prefix += bf16(bf16(acc) + shared) (kimi.py:325-329)
      bf16* prefix = reinterpret_cast<bf16*>(j.out) + o;
      const bf16* shared = reinterpret_cast<const bf16*>(j.aux) + o;
      float pv[8], sv[8], res[8];
      if (full) {
        unpack8(*reinterpret_cast<const uint4*>(prefix), pv);
        unpack8(*reinterpret_cast<const uint4*>(shared), sv);
      } else {
        for (int e = 0; e < 8; ++e) {
          pv[e] = rr + e < nrows ? bf2f(prefix[e]) : 0.0f;
          sv[e] = rr + e < nrows ? bf2f(shared[e]) : 0.0f;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) res[e] = pv[e] + round_bf(round_bf(v[e]) + sv[e]);
      if (full) {
        *reinterpret_cast<uint4*>(prefix) = pack8(res);
      } else {
        for (int e = 0; e < 8 && rr + e < nrows; ++e) prefix[e] = f2bf(res[e]);
      }
    } else if (epi == EPI_SIGMOID_F32 || epi == EPI_LOGITS) {
      float* d = reinterpret_cast<float*>(j.out) + o;
      float r[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = epi == EPI_LOGITS ? round_bf(v[e]) : sigmoidf_(v[e]);
      if (full) {
        *reinterpret_cast<float4*>(d) = make_float4(r[0], r[1], r[2], r[3]);
        *reinterpret_cast<float4*>(d + 4) = make_float4(r[4], r[5], r[6], r[7]);
      } else {
        for (int e = 0; e < 8 && rr + e < nrows; ++e) d[e] = r[e];
      }
    } else if (epi == EPI_STORE_BF16 || epi == EPI_LATENT) {
      bf16* d = reinterpret_cast<bf16*>(j.out) + o;
      const uint4 b = pack8(v);
      float r[8];
      unpack8(b, r);
      if (full) {
        *reinterpret_cast<uint4*>(d) = b;
      } else {
        for (int e = 0; e < 8 && rr + e < nrows; ++e) d[e] = f2bf(r[e]);
      }
      if (epi == EPI_LATENT) {   // FP16 copy of the bf16-rounded latent for the MXFP4 path
        __half* h = reinterpret_cast<__half*>(j.out2) + o;
        if (full) {
          __half2 hh[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) hh[e] = __floats2half2_rn(r[2 * e], r[2 * e + 1]);
          *reinterpret_cast<uint4*>(h) = *reinterpret_cast<const uint4*>(hh);
        } else {
          for (int e = 0; e < 8 && rr + e < nrows; ++e) h[e] = __float2half_rn(r[e]);
        }
      }
    }
  }
  __syncthreads();   // staging is rewritten by the next segment
}

// Run a list of BF16 jobs on the tensor cores (all CTAs, all threads). CTA-level stream-K: CTA c takes k-steps
// [U c / G, U (c + 1) / G) of the pass (U k-steps, G = min(CTAs, U)), so every CTA streams the same number of weight
// bytes; a block whose k-steps span several CTAs is finished by the last of them to arrive, which adds the
// partials in CTA order (each CTA keeps at most two: its first and its last block). Returns false when a
// bounded wait gave up (the error word is set; TMEM is released before returning).
template <int NT>
KK3_FN bool run_gemv_tc(const StepArgs& a, const GemvJob* jobs, int njobs, int parity, int bank = 0) {
  using Sh = TcGemvShape<NT>;
  constexpr int N = Sh::N, S = Sh::S, P = S - kTcgLag;   // P k-steps of copies in flight ahead of the MMAs
  static_assert(P >= 2, "too few stages for the refill lag");
  extern __shared__ __align__(1024) unsigned char kk3_dyn_smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned sbase = (unsigned)__cvta_generic_to_shared(kk3_dyn_smem);
  float* staging = reinterpret_cast<float*>(kk3_dyn_smem + S * Sh::kStage);
  unsigned char* ctl = kk3_dyn_smem + S * Sh::kStage + Sh::kStaging;
  const unsigned bar0 = sbase + S * Sh::kStage + Sh::kStaging;       // S mbarriers, 8 bytes each
  const unsigned tslot = bar0 + 8 * S;                              // TMEM base address (tcgen05.alloc)
  volatile int* flags = reinterpret_cast<volatile int*>(ctl + 96);  // [0] last arrival, [1] pass ok
  TcPlan& plan = *reinterpret_cast<TcPlan*>(ctl + 128);
  static_assert(128 + sizeof(TcPlan) <= Sh::kCtl, "control block");

  float* part_base = a.s.fix_part + bank * a.g.fix_bank;   // [G][2][N / 4][128] float4 partial blocks
  int* cnt_base = a.s.fix_cnt + bank * a.g.cnt_bank;
  if (tid == 0) {
    tc_plan(jobs, njobs, plan);
    for (int i = 0; i < S; ++i) mbar_init(bar0 + 8 * i, 1);
    fence_mbar_init();
    flags[1] = 1;
  }
  __syncthreads();
  // G = min(grid, U) participating CTAs, so that every range is non-empty: the CTAs between a block's first and
  // last owner are then exactly its contributors (an empty range would be counted but never arrive)
  const long long U = plan.total, G = (long long)gridDim.x < U ? (long long)gridDim.x : U;
  const long long rbeg = (long long)blockIdx.x < G ? U * blockIdx.x / G : U;
  const long long rend = (long long)blockIdx.x < G ? U * (blockIdx.x + 1) / G : U;
  const long long total_steps = rend - rbeg;
  if (total_steps <= 0) {
    __syncthreads();
    if (tid == 0)
      for (int i = 0; i < S; ++i) mbar_inval(bar0 + 8 * i);
    return true;
  }
  // TMEM for this pass only (released at its end); the allocation permit is kept, since every later pass of the
  // step allocates again (one CTA per SM, so the allocation never waits)
  if (warp == 0) tmem_alloc(tslot, Sh::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = *reinterpret_cast<volatile unsigned*>(ctl + 8 * S);
  const unsigned idesc = idesc_bf16_f32(N);
  const unsigned long long pol = l2_evict_first_policy();
  tc_stamp(a, 0);

  // ---- producer cursor over k-steps [rbeg, rend)
  TcPos pp = tc_locate(plan, rbeg);
  auto issue = [&](long long step) {
    const int st = (int)(step % S);
    const GemvJob& j = jobs[pp.job];
    const unsigned sa = sbase + st * Sh::kStage, sb = sa + kTcgStageA;
    // weights: 1024 16-byte chunks, two per thread; row r chunk c -> r * 128 + ((c ^ (r & 7)) << 4)
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int idx = tid + q * kThreads, r = idx >> 3, c = idx & 7;
      int row = pp.block * kTcgRows + r;
      row = row < j.rows ? row : j.rows - 1;
      const bf16* src = j.w + (size_t)row * j.K + (size_t)pp.ks * 64 + c * 8;
      asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;"
                   ::"r"(sa + r * 128 + ((c ^ (r & 7)) << 4)), "l"(src), "l"(pol) : "memory");
    }
    // activations: N rows x 8 chunks; rows past the batch are zero
    if (tid < N * 8) {
      const int r = tid >> 3, c = tid & 7;
      const unsigned dst = sb + r * 128 + ((c ^ (r & 7)) << 4);
      if (r < j.ncols) {
        const bf16* src = j.x + (size_t)r * j.ldx + (size_t)pp.ks * 64 + c * 8;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
      } else {
        st_shared_zero16(dst);
      }
    }
    if (++pp.ks == plan.ksteps[pp.job]) {
      pp.ks = 0;
      if (++pp.block == plan.blocks[pp.job]) {
        pp.block = 0;
        ++pp.job;
      }
    }
  };

  bool ok = true;
  long long issued = 0, last_commit = -1;
  for (; issued < P && issued < total_steps; ++issued) {
    issue(issued);
    cp_async_commit_g();
  }
  for (long long i = issued; i < P; ++i) cp_async_commit_g();   // keep the group count uniform

  // ---- consumer
  TcPos cp = tc_locate(plan, rbeg);
  bool seg_first = true;     // the segment being accumulated is this CTA's first
  int seg_k0 = cp.ks;        // its first k-step
  for (long long step = 0; step < total_steps; ++step) {
    if (issued < total_steps) {
      // the stage of k-step `issued` was last read by the MMAs of k-step issued - S = step - kTcgLag
      const long long prev = issued - S;
      if (prev >= 0 && !mbar_wait(a, bar0 + 8 * (int)(prev % S), (unsigned)((prev / S) & 1))) ok = false;
      issue(issued);
      ++issued;
    }
    cp_async_commit_g();
    cp_async_wait_g<P>();   // this thread's copies of `step` landed
    fence_async_smem();
    __syncthreads();
    if (step == 0) tc_stamp(a, 1);
    if (step + 1 == total_steps) tc_stamp(a, 2);
    const int st = (int)(step % S);
    if (tid == 0 && ok) {
      tc_fence_after();
      const unsigned sa = sbase + st * Sh::kStage, sb = sa + kTcgStageA;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16(tmem, sdesc_sw128(sa + kk * 32), sdesc_sw128(sb + kk * 32), idesc,
                  (cp.ks > seg_k0 || kk > 0) ? 1u : 0u);
      umma_commit(bar0 + 8 * st);
    }
    if (ok) last_commit = step;
    const int kend = plan.ksteps[cp.job];
    if (cp.ks + 1 == kend || step + 1 == total_steps) {
      // end of a segment: wait for its MMAs, read the accumulator (warps 0-3: TMEM lanes = block rows)
      if (!mbar_wait(a, bar0 + 8 * st, (unsigned)((step / S) & 1))) ok = false;
      tc_fence_after();
      const bool last_seg = step + 1 == total_steps;
      if (last_seg) tc_stamp(a, 3);
      const GemvJob& j = jobs[cp.job];
      const long long bstart = plan.ubase[cp.job] + (long long)cp.block * kend;
      const long long first = owner_of(bstart, U, G), lastc = owner_of(bstart + kend - 1, U, G);
      const bool whole = first == lastc;
      if (warp < 4 && ok) {
        const int row = warp * 32 + lane;
        float4* dst = reinterpret_cast<float4*>(part_base + ((size_t)blockIdx.x * 2 + (seg_first ? 0 : 1)) * kTcgRows * N);
#pragma unroll
        for (int h = 0; h < N / 16; ++h) {
          float v[16];
          tmem_ld16(tmem + ((unsigned)(warp * 32) << 16) + h * 16, v);
          tmem_ld_wait();
          if (whole) {   // staging is column-major: lanes (consecutive rows) hit consecutive banks
#pragma unroll
            for (int q = 0; q < 16; ++q) staging[(h * 16 + q) * Sh::kStagingStride + row] = v[q];
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)   // lanes write consecutive rows
              __stcg(dst + (size_t)(h * 4 + q) * kTcgRows + row, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
          }
        }
      }
      tc_fence_before();
      // the accumulator is free for the next segment and the partial / staging is written; a wait that gave up
      // on any thread stops the pass on every thread
      ok = __syncthreads_and(ok) != 0;
      if (last_seg) tc_stamp(a, 4);
      bool run_epi = ok && whole;
      if (ok && !whole) {
        const int blk_id = plan.bbase[cp.job] + cp.block;
        if (tid == 0) {
          __threadfence();
          const int old = atom_add_acq_rel_gpu(cnt_base + blk_id, 1);
          flags[0] = old == (int)(lastc - first);
        }
        __syncthreads();
        run_epi = flags[0] != 0;
        if (run_epi) {
          __threadfence();
          tc_reduce_block<NT>(part_base, staging, first, lastc, bstart, U, G);
          if (tid == 0) atomicExch(cnt_base + blk_id, 0);
          __syncthreads();
          if (last_seg) tc_stamp(a, 5);
        }
      }
      if (run_epi) {
        tc_epilogue_block<NT>(a, j, cp.block, staging, parity, reinterpret_cast<volatile int*>(ctl + Sh::kCtl - 64));
        if (last_seg) tc_stamp(a, 6);
      }
      seg_first = false;
      // next segment
      cp.ks = 0;
      if (++cp.block == plan.blocks[cp.job]) {
        cp.block = 0;
        ++cp.job;
      }
      seg_k0 = 0;
    } else {
      ++cp.ks;
    }
  }
  cp_async_wait_g<0>();
  // On success every MMA completed (each segment waited for its last commit). After a failed wait, thread 0
  // gives the MMAs it committed a bounded time to finish (they complete in order, so the last commit covers
  // them) before TMEM is released.
  if (!ok && tid == 0 && last_commit >= 0)
    mbar_wait_for(bar0 + 8 * (int)(last_commit % S), (unsigned)((last_commit / S) & 1), 1000000ull);
  tc_fence_before();
  ok = __syncthreads_and(ok) != 0;
  if (!ok && tid == 0) flags[1] = 0;
  if (warp == 0) tmem_dealloc(tmem, Sh::kTmemCols);
  if (tid == 0)
    for (int i = 0; i < S; ++i) mbar_inval(bar0 + 8 * i);
  __syncthreads();
  tc_stamp(a, 7);
  return flags[1] != 0;
}

}  // namespace kk3
