// kk3_tc_attn.cuh - the MLA split-K attention of the decode step (kimi.py:274-280, absorbed latent form) on the
// 5th-generation tensor cores (tcgen05.mma kind::f16, sm_100a).
//
// An item is (batch row b, chunk of its attended positions, head group, value half). The partial it writes is the
// warp-level engine's (mla_attend_item, kk3_phases.cuh): per head (m, l, O) with O = sum_t exp(s_t - m) V_t and
// l = sum_t exp(s_t - m), which the combine phase merges over the chunks. Per 32-position sub-tile:
//  - all threads copy the cached rows (512 latent + 64 rope dims, bf16) with 16-byte cp.async into a
//    128-byte-swizzled tile [9 blocks of 64 dims][32 positions][128 B] (the new token's rows are stored directly,
//    positions past the attended sequence are zero), in a ring of NS stages running NS - 2 sub-tiles ahead;
//  - thread 0 issues S = Q K^T: M = 128 (the group's head rows; rows past them are never read back), N = 32
//    positions, K = 576 in 36 steps of 16, FP32 into one of two TMEM column buffers;
//  - warps 0-3 (thread = head row = its TMEM lane) read their row of S, mask positions past the chunk and run the
//    online softmax in registers: each thread owns its head's whole row, so there are no shuffles. The running
//    maximum moves only when a score exceeds it by more than kTaSlack, so the FP32 accumulator O in TMEM is
//    rescaled rarely (the probabilities exp(s - m) then stay below e^kTaSlack; O / l is the same quotient). The
//    BF16 probabilities go to shared memory in the MMA's K-major layout;
//  - thread 0 issues O += P V over this item's 256 value dims: the same shared tile read as an MN-major B operand
//    (N = 256 dims, K = 32 positions), so the cache rows are staged once for both products.
// The 512 FP32 columns of a whole O do not fit in TMEM next to S, so the two halves of the value dims are
// separate, adjacent items (the second CTA's copies of the same cache rows come from L2); both compute the same S.
// Every wait is bounded; TMEM is held for the phase and released at its end.
//
// Selected with kk3_set_attn_engine(KK3_ATTN_TC); the warp-level engine stays the default because it is faster at
// this step's head counts (12-96 per rank). Measured in the step (B200): a sub-tile takes ~4.7 us, of which the 36
// N = 32 products of S take ~1.8 us (each instruction re-reads the 4 KB query block from shared memory, so small N
// runs far below the tensor pipe's rate) and the serial softmax ~1.9 us; with the value halves an item also walks
// twice the sub-tiles. mla_attend at dev-l4: 329 us against 146 us for the warp-level engine.
#pragma once
#include "kk3_phases.cuh"
#include "kk3_tc_gemv.cuh"

namespace kk3 {

constexpr int kTaDims = 576;                       // 512 latent + 64 rope dims per cached position
constexpr int kTaBlocks = kTaDims / 64;            // 64-dim (128-byte) blocks per position
constexpr int kTaBlock = kMlaPos * 128;            // bytes of one 64-dim block of a sub-tile (32 rows)
constexpr int kTaStage = kTaBlocks * kTaBlock;     // 36864 bytes: one 32-position sub-tile
constexpr int kTaP = 128 * 128;                    // BF16 probabilities: 128 rows x 128 bytes (32 positions used)
constexpr int kTaCtl = 1024;                       // mbarriers and the TMEM address
constexpr int kTaMaxStages = 6;
constexpr int kTaTmemCols = 512;
constexpr int kTaO = 256;                          // TMEM column of O (256 columns); S buffers at columns 0 and 32
constexpr float kTaSlack = 8.0f;                   // the running maximum moves when exceeded by more than this

// Query bytes of a group of hg head rows (hg a multiple of 8, so that every 64-dim block starts on a 1024-byte
// swizzle atom), and the ring depth that fits the step kernel's dynamic shared memory next to it.
__host__ __device__ inline int ta_qbytes(int hg) { return kTaBlocks * hg * 128; }
__host__ __device__ inline int ta_stages(int hg) {
  const int ns = (kExpSmem - ta_qbytes(hg) - kTaP - kTaCtl) / kTaStage;
  return ns > kTaMaxStages ? kTaMaxStages : ns;
}

// Instruction descriptor of the P V product: kind::f16, D = F32, A = B = BF16, M = 128, N = 256, A K-major and
// B MN-major (bit 16).
KK3_DEV unsigned ta_idesc_pv() { return idesc_bf16_f32(256) | (1u << 16); }
// Shared-memory descriptor of an MN-major operand with the 128-byte swizzle: 64-element MN blocks of 8 K-rows
// (1024-byte atoms); `lbo` bytes between MN blocks (leading byte offset), 1024 bytes between 8-row K groups.
KK3_DEV unsigned long long sdesc_sw128_mn(unsigned addr, unsigned lbo) {
  return (unsigned long long)((addr & 0x3ffffu) >> 4) | ((unsigned long long)(lbo >> 4) << 16) |
         ((unsigned long long)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// 32 TMEM lanes (one per thread of the warp) x 16 consecutive 32-bit columns
KK3_DEV void tmem_st16(unsigned taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
      : "memory");
}
KK3_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// named barrier of the four softmax warps (warps 0-3; barrier 0 is __syncthreads)
KK3_DEV void ta_softmax_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
KK3_DEV void st_shared_v4(unsigned addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
KK3_DEV void cp_async16_u32(unsigned dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
KK3_DEV void cp_async16_pol(unsigned dst, const void* src, unsigned long long pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(pol)
               : "memory");
}

// Stage positions [t0, t0 + 32) of the item's sequence into the swizzled tile at `dst` (this thread's pieces):
// piece (row tl, 16-byte chunk q of 72) goes to block q / 8, row tl, chunk (q % 8) ^ (tl % 8).
KK3_DEV void ta_stage(const MlaSrc& src, int t0, int T, unsigned dst) {
#pragma unroll
  for (int j = 0; j < kMlaPiecesPerThread; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i >= kMlaPieces) break;
    const int tl = i / 72, q = i - tl * 72, t = t0 + tl;
    const unsigned d = dst + (q >> 3) * kTaBlock + tl * 128 + (((q & 7) ^ (tl & 7)) << 4);
    if (t < src.ncache) {
      cp_async16_pol(d, q < 64 ? src.kv + (size_t)t * src.kr + q * 8 : src.pe + (size_t)t * src.rd + (q - 64) * 8,
                     src.pol);
    } else if (t < T) {
      st_shared_v4(d, ld_act16(q < 64 ? src.kvw + q * 8 : src.pew + (q - 64) * 8));
    } else {
      st_shared_zero16(d);
    }
  }
}

// Shared-memory addresses of the phase (Q at the start of the dynamic shared memory, then the ring, P, control).
struct TaSmem {
  unsigned q, ring, p, bar_s, bar_o, bar_st, tslot;
};

// One item (all threads). `gs` counts the sub-tiles this CTA ran before in the phase: ring slot and mbarrier
// parities continue across items. `last_pv`: thread 0's last committed P V sub-tile (for the cleanup after a
// failed wait). Returns false (the same on every thread) when a bounded wait gave up.
template <int NS>
KK3_DEV bool ta_item(const StepArgs& a, int layer, int midx, int b, int chunk, int grp, int half, unsigned& gs,
                     long long& last_pv, const TaSmem& m, unsigned tmem, int ph) {
  constexpr int PA = NS - 2;   // sub-tiles of copies in flight ahead of the MMAs (a slot is refilled two later)
  static_assert(PA >= 2, "ring too shallow");
  const Geo& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hg = g.mla_hg, QB = hg * 128;
  const int T = mla_row_len(a, b) + 1;
  const int p0 = chunk * g.mla_chunk_len;
  const int p1 = p0 + g.mla_chunk_len < T ? p0 + g.mla_chunk_len : T;
  const int nsub = (p1 - p0 + kMlaPos - 1) / kMlaPos;
  const int h0 = grp * hg;
  const bool stamp = ph >= 0 && gs == 0 && blockIdx.x == 0 && tid == 0;   // sub-phase stamps of one item
  if (stamp) sub_stamp(a, ph, 0);
  MlaSrc src;
  src.kv = lptr<bf16>(a, layer, KK3_MLA_KV_CACHE) + (size_t)b * g.ctx * g.kr;
  src.pe = lptr<bf16>(a, layer, KK3_MLA_PE_CACHE) + (size_t)b * g.ctx * g.rd;
  src.kvw = gout<bf16>(a, KK3_OUT_KV_WRITE) + ((size_t)midx * g.B + b) * g.kr;
  src.pew = gout<bf16>(a, KK3_OUT_PE_WRITE) + ((size_t)midx * g.B + b) * g.rd;
  src.ncache = mla_row_len(a, b);
  src.pol = l2_evict_first_policy();
  src.kr = g.kr;
  src.rd = g.rd;
  // Q rows of heads h0 .. h0 + hg - 1: absorbed (512) | q rope (64), zero past the heads; in the copy group of
  // the first sub-tile (the MMAs of the previous item, which read Q, completed before it ended)
  for (int i = tid; i < hg * 72; i += kThreads) {
    const int hh = i / 72, q = i - hh * 72, h = h0 + hh;
    const unsigned d = m.q + (q >> 3) * QB + hh * 128 + (((q & 7) ^ (hh & 7)) << 4);
    if (h < g.hr) {
      cp_async16_u32(d, q < 64 ? a.s.absorbed + ((size_t)b * g.hr + h) * g.kr + q * 8
                               : a.s.mla_q + ((size_t)b * g.hr + h) * (g.nr + g.rd) + g.nr + (q - 64) * 8);
    } else {
      st_shared_zero16(d);
    }
  }
  bool ok = true;
  // the slot of global sub-tile u was last read by the MMAs of sub-tile u - NS (committed to its mbarrier)
  auto slot_free = [&](unsigned u) {
    if (u >= (unsigned)NS && !mbar_wait(a, m.bar_st + 8 * (u % NS), ((u - NS) / NS) & 1u)) ok = false;
  };
  for (int s = 0; s < PA; ++s) {
    if (s < nsub) {
      slot_free(gs + s);
      if (ok) ta_stage(src, p0 + s * kMlaPos, p1, m.ring + ((gs + s) % NS) * kTaStage);
    }
    cp_async_commit_g();
  }
  if (stamp) sub_stamp(a, ph, 1);

  const float scale = rsqrtf((float)(g.nr + g.rd));
  const unsigned id_s = idesc_bf16_f32(kMlaPos), id_pv = ta_idesc_pv();
  const int r = (warp & 3) * 32 + lane;                 // softmax warps: head row = TMEM lane
  const unsigned tlane = (unsigned)((warp & 3) * 32) << 16;
  const bool row_ok = r < hg && h0 + r < g.hr;
  float m_run = -INFINITY, l_run = 0.0f;
  for (int s = 0; s < nsub; ++s) {
    const unsigned u = gs + s, st = u % NS;
    if (s + PA < nsub) {
      slot_free(u + PA);
      if (ok) ta_stage(src, p0 + (s + PA) * kMlaPos, p1, m.ring + ((u + PA) % NS) * kTaStage);
    }
    cp_async_commit_g();
    cp_async_wait_g<PA>();   // this thread's copies of sub-tile s (and of Q) landed
    fence_async_smem();      // ... and are visible to the tensor core's (async proxy) reads
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    if (stamp && s < 2) sub_stamp(a, ph, 2 + 4 * s);
    const unsigned stg = m.ring + st * kTaStage, s_col = tmem + (u & 1u) * kMlaPos;
    if (tid == 0) {
      tc_fence_after();
#pragma unroll 1
      for (int d = 0; d < kTaBlocks; ++d)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(s_col, sdesc_sw128(m.q + d * QB + kk * 32), sdesc_sw128(stg + d * kTaBlock + kk * 32), id_s,
                    (d | kk) ? 1u : 0u);
      umma_commit(m.bar_s + 8 * (u & 1u));
    }
    if (warp < 4) {
      if (!mbar_wait(a, m.bar_s + 8 * (u & 1u), (u >> 1) & 1u)) ok = false;
      tc_fence_after();
      if (stamp && s < 2) sub_stamp(a, ph, 3 + 4 * s);
      float sv[32];
      {
        float v0[16], v1[16];
        tmem_ld16(s_col + tlane, v0);
        tmem_ld16(s_col + tlane + 16, v1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          sv[j] = v0[j];
          sv[16 + j] = v1[j];
        }
      }
      const int t0 = p0 + s * kMlaPos;
      float mloc = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        sv[j] = row_ok && t0 + j < p1 ? sv[j] * scale : -INFINITY;   // rows past the heads: no probabilities
        mloc = fmaxf(mloc, sv[j]);
      }
      // false when mloc is -inf; true for a finite mloc while m_run is still -inf
      const bool move = mloc > m_run + kTaSlack;
      const float mnew = move ? mloc : m_run;
      const float alpha = move ? (m_run == -INFINITY ? 0.0f : expf(m_run - mnew)) : 1.0f;
      float psum = 0.0f;
      unsigned pw[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float pa = sv[j] == -INFINITY ? 0.0f : expf(sv[j] - mnew);
        const float pb = sv[j + 1] == -INFINITY ? 0.0f : expf(sv[j + 1] - mnew);
        psum += pa;
        psum += pb;
        pw[j >> 1] = pack_bf2(pa, pb);
      }
      l_run = l_run * alpha + psum;
      m_run = mnew;
      if (s > 0) {
        // the previous P V finished: P may be rewritten and O is stable
        if (!mbar_wait(a, m.bar_o, (u - 1) & 1u)) ok = false;
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {   // only head rows can move (the others stay at -inf)
#pragma unroll 1
          for (int c = 0; c < 16; ++c) {
            float v[16];
            tmem_ld16(tmem + kTaO + tlane + c * 16, v);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] *= alpha;
            tmem_st16(tmem + kTaO + tlane + c * 16, v);
          }
          tmem_st_wait();
        }
      }
      const unsigned prow = m.p + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        st_shared_v4(prow + ((c ^ (r & 7)) << 4), make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]));
      fence_async_smem();
      tc_fence_before();
      ta_softmax_sync();
      if (stamp && s < 2) sub_stamp(a, ph, 4 + 4 * s);
      if (tid == 0 && ok) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 2; ++kk)
          umma_bf16(tmem + kTaO, sdesc_sw128(m.p + kk * 32),
                    sdesc_sw128_mn(stg + 4 * half * kTaBlock + kk * 16 * 128, kTaBlock), id_pv,
                    (s > 0 || kk > 0) ? 1u : 0u);
        umma_commit(m.bar_o);
        umma_commit(m.bar_st + 8 * st);
        last_pv = u;
        if (stamp && s < 2) sub_stamp(a, ph, 5 + 4 * s);
      }
    }
  }
  if (ok && nsub > 0) {
    // the item's last P V (its commit covers every MMA before it): O is final, Q and the ring may be reused
    if (!mbar_wait(a, m.bar_o, (gs + nsub - 1) & 1u)) ok = false;
    tc_fence_after();
    if (warp < 4 && ok) {
      float* base = a.s.mla_part + (((size_t)b * g.mla_chunks + chunk) * g.hr + (row_ok ? h0 + r : 0)) * (g.kr + 2);
#pragma unroll 1
      for (int c = 0; c < 16; ++c) {
        float v[16];
        tmem_ld16(tmem + kTaO + tlane + c * 16, v);
        tmem_ld_wait();
        if (row_ok) {
          float2* o = reinterpret_cast<float2*>(base + 2 + half * 256 + c * 16);   // 8-byte aligned ((kr + 2) even)
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] = make_float2(v[2 * e], v[2 * e + 1]);
        }
      }
      if (row_ok && half == 0) {
        base[0] = m_run;
        base[1] = l_run;
      }
    }
    tc_fence_before();
  }
  ok = __syncthreads_and(ok) != 0;   // O was read before the next item's first P V overwrites it
  if (stamp) {
    sub_stamp(a, ph, 10);
    sub_stamp(a, ph, 11, (unsigned long long)nsub);
  }
  gs += (unsigned)nsub;
  return ok;
}

// The attention phase on the tensor cores (all threads of every CTA). Items: (row, chunk, group, half), the
// halves and then the groups of one chunk adjacent. Returns false when a bounded wait gave up (the error word is
// set; TMEM is released first).
template <int NS>
KK3_DEV bool ta_phase(const StepArgs& a, int layer, int midx, int ph) {
  extern __shared__ __align__(1024) unsigned char kk3_dyn_smem[];
  const Geo& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5;
  int total = 0;
#pragma unroll 1
  for (int b = 0; b < g.B; ++b) total += mla_row_chunks(a, b);
  total *= g.mla_groups * 2;
  if ((int)blockIdx.x >= total) return true;   // the same for every thread of the CTA
  TaSmem m;
  m.q = (unsigned)__cvta_generic_to_shared(kk3_dyn_smem);
  m.ring = m.q + ta_qbytes(g.mla_hg);
  m.p = m.ring + NS * kTaStage;
  m.bar_s = m.p + kTaP;            // two mbarriers (S buffers)
  m.bar_o = m.bar_s + 16;          // P V commits
  m.bar_st = m.bar_o + 8;          // NS mbarriers (ring slots)
  m.tslot = m.bar_s + 128;         // TMEM base address (tcgen05.alloc)
  if (tid == 0) {
    for (int i = 0; i < 3 + NS; ++i) mbar_init(m.bar_s + 8 * i, 1);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(m.tslot, kTaTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = *reinterpret_cast<volatile unsigned*>(kk3_dyn_smem + (m.tslot - m.q));
  unsigned gs = 0;
  long long last_pv = -1;
  bool ok = true;
#pragma unroll 1
  for (int it = blockIdx.x; it < total; it += gridDim.x) {
    const int half = it & 1;
    int rest = it >> 1;
    const int grp = rest % g.mla_groups;
    rest /= g.mla_groups;
    int b = 0;
    for (; b < g.B; ++b) {
      const int n = mla_row_chunks(a, b);
      if (rest < n) break;
      rest -= n;
    }
    ok = ta_item<NS>(a, layer, midx, b, rest, grp, half, gs, last_pv, m, tmem, ph);
    if (!ok) break;
  }
  cp_async_wait_g<0>();
  // On success every MMA completed (each item waited for its last commit). After a failed wait, thread 0 gives
  // the MMAs it committed a bounded time to finish (they complete in order) before TMEM is released.
  if (!ok && tid == 0 && last_pv >= 0) mbar_wait_for(m.bar_o, (unsigned)(last_pv & 1), 1000000ull);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTaTmemCols);
  if (tid == 0)
    for (int i = 0; i < 3 + NS; ++i) mbar_inval(m.bar_s + 8 * i);
  __syncthreads();
  return ok;
}

KK3_FN bool mla_attend_tc(const StepArgs& a, int layer, int midx, int ph) {
  switch (a.g.mla_ns) {
    case 4: return ta_phase<4>(a, layer, midx, ph);
    case 5: return ta_phase<5>(a, layer, midx, ph);
    default: return ta_phase<6>(a, layer, midx, ph);
  }
}

}  // namespace kk3
