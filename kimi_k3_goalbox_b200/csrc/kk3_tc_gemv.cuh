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
//  - a stage is refilled only after the mbarrier of the MMAs that read it completed, three k-steps later, so
//    the MMA latency stays off the copy path; the copies run S - 3 k-steps ahead of the MMAs, across blocks.
// At the end of a segment (the CTA's k-steps of one block) warps 0-3 read the accumulator (TMEM lane = block
// row) with tcgen05.ld. A block done by one CTA goes straight to the epilogue; otherwise each contributor
// writes its FP32 partial to the stream-K bank and the last to arrive sums them in CTA order (deterministic)
// before the epilogue. The epilogue
// is the GEMV engine's: the 128 x N block is staged in shared memory and eight warps each run
// gemv_epilogue on one 16-row tile in the mma.sync fragment layout, so every fused epilogue (exchange
// stores, situ pairs, logits keys, ...) is shared with the mma.sync path.
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
  static constexpr int kStagingStride = N + 4;                   // floats per staged result row
  static constexpr int kStaging = kTcgRows * kStagingStride * 4;
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

constexpr int kTcgLag = 3;   // a stage is refilled once the MMAs of 3 k-steps ago completed

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
          if (whole) {
            float* srow = staging + row * Sh::kStagingStride + h * 16;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<float4*>(srow + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
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
          // sum the contributors' partials in CTA order (their first or last segment)
          const int ncon = (int)(lastc - first) + 1;
          for (int e = tid; e < kTcgRows * N / 4; e += kThreads) {
            const int q = e / kTcgRows, row = e - q * kTcgRows;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            for (int k0 = 0; k0 < ncon; k0 += 4) {
              float4 v[4];
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                v[t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                if (k0 + t < ncon) {
                  const long long c = first + k0 + t;
                  const int slot = (U * c / G >= bstart) ? 0 : 1;
                  v[t] = __ldcg(reinterpret_cast<const float4*>(part_base + ((size_t)c * 2 + slot) * kTcgRows * N) +
                                (size_t)q * kTcgRows + row);
                }
              }
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                acc.x += v[t].x; acc.y += v[t].y; acc.z += v[t].z; acc.w += v[t].w;
              }
            }
            *reinterpret_cast<float4*>(staging + row * Sh::kStagingStride + 4 * q) = acc;
          }
          if (tid == 0) atomicExch(cnt_base + blk_id, 0);
          __syncthreads();
        }
      }
      if (run_epi) {
        // eight warps, one 16-row tile each, in the mma.sync fragment layout of gemv_epilogue
        const int wt = warp & 7, tile = cp.block * 8 + wt;
        if (warp < 8 && tile * 16 < j.rows) {
          const int r = lane >> 2, c = lane & 3;
          float acc[1][NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              acc[0][nt][i] = staging[(wt * 16 + r + 8 * (i >> 1)) * Sh::kStagingStride + nt * 8 + 2 * c + (i & 1)];
          gemv_epilogue<NT, 1>(a, j, tile, acc, parity);
        }
        __syncthreads();   // staging is rewritten by the next segment
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
  return flags[1] != 0;
}

}  // namespace kk3
