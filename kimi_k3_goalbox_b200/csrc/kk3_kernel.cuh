// kk3_kernel.cuh - the persistent cooperative kernel computing one Kimi K3 decode step per rank on sm_100a.
//
// The kernel walks the step as a fixed program of grid-wide phases separated by bounded grid barriers
// (the reference's per-op torch calls, megabench/tasks/kimi.py:230-340, become phases of one launch):
//   embed | per layer: [attn prologue | attn projections | KDA or MLA (5 phases) | o proj | mlp prologue |
//   dense FFN (2) or MoE (router+latent+shared | routing ∥ shared down | experts gate/up | experts down |
//   combine | latent up)] | head prologue | lm head | argmax.
// Tensor-parallel reductions are one-shot stores into peers' exchange buffers plus per-row release flags.

#pragma once

#include "kk3_phases.cuh"

namespace kk3 {

KK3_DEV bool layer_is_mla(const Geo& g, int l) { return ((l + 1) % 4 == 0) || (l == g.L - 1); }

enum Pending : int { PEND_NONE = 0, PEND_EMBED, PEND_DENSE };

// ---- row phases ------------------------------------------------------------------------------------

KK3_DEV void phase_embed(const StepArgs& a, unsigned seq, int parity, float* fsm) {
  const Geo& g = a.g;
  const long long* tok = gptr<long long>(a, KK3_TOKEN);
  const bf16* emb = gptr<bf16>(a, KK3_EMBED);
  long long* out_ids = gout<long long>(a, KK3_OUT_EXPERT_IDS);
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    const long long t = tok[b] - (long long)g.rank * g.V;
    const bool mine = t >= 0 && t < g.V;
    const bf16* row = emb + (size_t)(mine ? t : 0) * g.h;
    const bf16 zero = f2bf(0.0f);
    if (g.tp == 1) {
      for (int e = threadIdx.x; e < g.h; e += kThreads) a.s.prefix[(size_t)b * g.h + e] = mine ? row[e] : zero;
    } else {
      const size_t off = ((size_t)g.rank * g.B + b) * g.h;
      for (int dst = 0; dst < g.tp; ++dst) {
        bf16* reg = reinterpret_cast<bf16*>(a.comm.base[dst] + a.comm.data_off[parity] + a.comm.att_off);
        for (int e = threadIdx.x; e < g.h; e += kThreads) reg[off + e] = mine ? row[e] : zero;
      }
      xch_signal_row(a, b, seq);
    }
    // dense layers report -1 expert ids (kimi.py:305)
    for (int l = 0; l < g.first_dense && l < g.L; ++l)
      for (int j = threadIdx.x; j < g.K; j += kThreads) out_ids[((size_t)l * g.B + b) * g.K + j] = -1;
  }
  (void)fsm;
}

// finish a pending exchange into prefix (embedding: assign; dense FFN: add), then the attention prologue
KK3_DEV bool phase_attn_prologue(const StepArgs& a, int layer, int nb, int pending, bool need_signal, unsigned seq,
                                 int parity, float* fsm) {
  const Geo& g = a.g;
  float* red = fsm;
  float* hbuf = fsm + 512;
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (pending != PEND_NONE) {
      if (g.tp > 1) {
        if (need_signal) xch_signal_row(a, b, seq);
        if (!xch_wait_row(a, b, seq)) return false;
      }
      bf16* pre = a.s.prefix + (size_t)b * g.h;
      for (int e = threadIdx.x; e < g.h; e += kThreads) {
        float v;
        if (g.tp == 1 && pending == PEND_EMBED) {
          v = bf2f(pre[e]);
        } else {
          v = xch_sum_bf16(a, parity, a.comm.att_off, b, g.h, e);
          if (pending == PEND_DENSE) v = round_bf(bf2f(pre[e]) + v);
        }
        pre[e] = f2bf(v);
      }
      __syncthreads();
    }
    mix_and_norm(a, b, nb, gptr<bf16>(a, KK3_ATTENTION_RES_NORM) + (size_t)layer * g.h,
                 gptr<bf16>(a, KK3_ATTENTION_RES_PROJ) + (size_t)layer * g.h, gptr<bf16>(a, KK3_LN1) + (size_t)layer * g.h,
                 1e-5f, a.s.xa + (size_t)b * g.h, hbuf, red);
    if (layer % g.bs == 0) {
      bf16* dst = a.s.blocks + ((size_t)nb * g.B + b) * g.h;
      for (int e = threadIdx.x; e < g.h; e += kThreads) dst[e] = a.s.prefix[(size_t)b * g.h + e];
    }
    __syncthreads();
  }
  return true;
}

// fold a pending exchange into prefix without a following norm (only when the last layer is dense)
KK3_DEV bool phase_fold_pending(const StepArgs& a, int pending, bool need_signal, unsigned seq, int parity) {
  const Geo& g = a.g;
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (g.tp > 1) {
      if (need_signal) xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
    }
    bf16* pre = a.s.prefix + (size_t)b * g.h;
    for (int e = threadIdx.x; e < g.h; e += kThreads) {
      const float v = xch_sum_bf16(a, parity, a.comm.att_off, b, g.h, e);
      pre[e] = f2bf(pending == PEND_DENSE ? round_bf(bf2f(pre[e]) + v) : v);
    }
    __syncthreads();
  }
  return true;
}

// attention exchange -> prefix (assign right after a block push, else add), then the MLP prologue
KK3_DEV bool phase_mlp_prologue(const StepArgs& a, int layer, int nb_after, unsigned seq, int parity, float* fsm) {
  const Geo& g = a.g;
  float* red = fsm;
  float* hbuf = fsm + 512;
  const bool assign = (layer % g.bs) == 0;
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (g.tp > 1) {
      xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
    }
    bf16* pre = a.s.prefix + (size_t)b * g.h;
    for (int e = threadIdx.x; e < g.h; e += kThreads) {
      const float att = xch_sum_bf16(a, parity, a.comm.att_off, b, g.h, e);
      pre[e] = f2bf(assign ? att : round_bf(bf2f(pre[e]) + att));
    }
    __syncthreads();
    mix_and_norm(a, b, nb_after, gptr<bf16>(a, KK3_MLP_RES_NORM) + (size_t)layer * g.h,
                 gptr<bf16>(a, KK3_MLP_RES_PROJ) + (size_t)layer * g.h, gptr<bf16>(a, KK3_LN2) + (size_t)layer * g.h, 1e-5f,
                 a.s.xm + (size_t)b * g.h, hbuf, red);
  }
  return true;
}

// MLA row prologue: q_a norm, latent norm (-> kv_write), rope part (-> pe_write)  (kimi.py:265-270)
KK3_DEV void phase_mla_rows(const StepArgs& a, int layer, int midx, float* fsm) {
  const Geo& g = a.g;
  const bf16* qa = a.s.qkv;
  const bf16* ka = a.s.qkv + (size_t)g.B * g.qr;
  bf16* kvw = gout<bf16>(a, KK3_OUT_KV_WRITE) + (size_t)midx * g.B * g.kr;
  bf16* pew = gout<bf16>(a, KK3_OUT_PE_WRITE) + (size_t)midx * g.B * g.rd;
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    rms_row(qa + (size_t)b * g.qr, lptr<bf16>(a, layer, KK3_MLA_QN), g.qr, 1e-6f, a.s.mla_qan + (size_t)b * g.qr, fsm);
    rms_row(ka + (size_t)b * (g.kr + g.rd), lptr<bf16>(a, layer, KK3_MLA_KN), g.kr, 1e-6f, kvw + (size_t)b * g.kr, fsm);
    for (int e = threadIdx.x; e < g.rd; e += kThreads) pew[(size_t)b * g.rd + e] = ka[(size_t)b * (g.kr + g.rd) + g.kr + e];
    __syncthreads();
  }
}

// MoE combine: expert_sum (slot order = ascending expert id, kimi.py:319-323), TP sum (:324),
// latent_norm (:325) -> x3; shared-expert TP sum (:326) -> shared_red
KK3_DEV bool phase_moe_combine(const StepArgs& a, int layer, unsigned seq, int parity, float* fsm) {
  const Geo& g = a.g;
  float* red = fsm;
  float* tot = fsm + 512;   // [lh]
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    const float* w = a.s.route_w + (size_t)b * g.K;
    for (int e = threadIdx.x; e < g.lh; e += kThreads) {
      float acc = 0.0f;
      for (int j = 0; j < g.K; ++j) acc += bf2f(a.s.out_slot[((size_t)b * g.K + j) * g.lh + e]) * w[j];
      tot[e] = acc;
      a.s.expert_sum[(size_t)b * g.lh + e] = acc;
    }
    if (g.tp > 1) {
      const size_t off = ((size_t)g.rank * g.B + b) * g.lh;
      for (int dst = 0; dst < g.tp; ++dst) {
        float* reg = reinterpret_cast<float*>(a.comm.base[dst] + a.comm.data_off[parity] + a.comm.exp_off);
        for (int e = threadIdx.x; e < g.lh; e += kThreads) reg[off + e] = tot[e];
      }
      xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
      const float* reg = xlocal<float>(a, parity, a.comm.exp_off);
      for (int e = threadIdx.x; e < g.lh; e += kThreads) {
        float acc = 0.0f;
        for (int src = 0; src < g.tp; ++src) acc += reg[((size_t)src * g.B + b) * g.lh + e];
        tot[e] = acc;
      }
    }
    __syncthreads();
    // x3 = rms(bf16(total), latent_norm)
    float ss = 0.0f;
    for (int e = threadIdx.x; e < g.lh; e += kThreads) {
      const float v = round_bf(tot[e]);
      tot[e] = v;
      ss += v * v;
    }
    const float s = block_sum(ss, red);
    const float rs = rsqrtf(s / (float)g.lh + 1e-5f);
    const bf16* ln = lptr<bf16>(a, layer, KK3_MOE_LATENT_NORM);
    for (int e = threadIdx.x; e < g.lh; e += kThreads)
      a.s.x3[(size_t)b * g.lh + e] = f2bf(round_bf(tot[e] * rs) * bf2f(ln[e]));
    for (int e = threadIdx.x; e < g.h; e += kThreads)
      a.s.shared_red[(size_t)b * g.h + e] = f2bf(xch_sum_bf16(a, parity, a.comm.shd_off, b, g.h, e));
    __syncthreads();
  }
  return true;
}

KK3_DEV void phase_head_prologue(const StepArgs& a, int nb, float* fsm) {
  const Geo& g = a.g;
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    mix_and_norm(a, b, nb, gptr<bf16>(a, KK3_OUTPUT_RES_NORM), gptr<bf16>(a, KK3_OUTPUT_RES_PROJ),
                 gptr<bf16>(a, KK3_FNORM), 1e-5f, a.s.xa + (size_t)b * g.h, fsm + 512, fsm);
    if (threadIdx.x == 0) a.s.argmax_key[b] = 0ull;
  }
}

KK3_DEV bool phase_argmax(const StepArgs& a, unsigned seq, int parity) {
  const Geo& g = a.g;
  long long* next = gout<long long>(a, KK3_OUT_NEXT_TOKEN);
  long long* len = gout<long long>(a, KK3_OUT_CACHE_LENGTH);
  const bool* reset = gptr<bool>(a, KK3_RESET);
  __shared__ unsigned long long best;
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (threadIdx.x == 0) best = *reinterpret_cast<volatile unsigned long long*>(a.s.argmax_key + b);
    __syncthreads();
    if (g.tp > 1) {
      const size_t off = (size_t)g.rank * g.B + b;
      if ((int)threadIdx.x < g.tp) {
        unsigned long long* reg =
            reinterpret_cast<unsigned long long*>(a.comm.base[threadIdx.x] + a.comm.data_off[parity] + a.comm.key_off);
        reg[off] = best;
      }
      xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
      if (threadIdx.x == 0) {
        const unsigned long long* reg = xlocal<unsigned long long>(a, parity, a.comm.key_off);
        unsigned long long m = 0ull;
        for (int src = 0; src < g.tp; ++src) {
          const unsigned long long k = reg[(size_t)src * g.B + b];
          m = k > m ? k : m;
        }
        best = m;
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      next[b] = (long long)(0xffffffffu - (unsigned)(best & 0xffffffffull));
      len[b] = reset[b] ? 1 : (long long)g.ctx + 1;
    }
    __syncthreads();
  }
  return true;
}

// ---- the kernel -------------------------------------------------------------------------------------

template <int NT>
__global__ void __launch_bounds__(kThreads, 1) kk3_step_kernel(const __grid_constant__ StepArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const Geo& g = a.g;
  float* fsm = reinterpret_cast<float*>(smem);
  int phase = 0;
  unsigned xi = 0;
  const unsigned seq0 = a.epoch * 1024u;
#define KK3_RUN (phase >= a.start_phase)
#define KK3_PHASE_END()                                                                      \
  do {                                                                                       \
    if (KK3_RUN && !grid_sync(a)) return;                                                    \
    ++phase;                                                                                 \
    if (blockIdx.x == 0 && threadIdx.x == 0 && phase <= kMaxPhases) a.s.phase_ts[phase] = globaltimer(); \
    if (phase == a.stop_phase) return;                                                       \
  } while (0)

  if (blockIdx.x == 0 && threadIdx.x == 0) a.s.phase_ts[0] = globaltimer();
  // embedding (kimi.py:249-252)
  if (KK3_RUN) phase_embed(a, seq0 + xi, xi & 1, fsm);
  int pending = PEND_EMBED;
  bool pend_signal = false;
  unsigned pend_x = xi++;
  KK3_PHASE_END();

  int nb = 0, kidx = 0, midx = 0;
  for (int l = 0; l < g.L; ++l) {
    const bool mla = layer_is_mla(g, l);
    // attention prologue (kimi.py:257-262)
    if (KK3_RUN && !phase_attn_prologue(a, l, nb, pending, pend_signal, seq0 + pend_x, pend_x & 1, fsm)) return;
    pending = PEND_NONE;
    if (l % g.bs == 0) ++nb;
    KK3_PHASE_END();
    if (!mla) {
      // KDA projections (kimi.py:285, :290-291, :298)
      GemvJob jobs[6] = {};
      const bf16* wq[4] = {lptr<bf16>(a, l, KK3_KDA_Q), lptr<bf16>(a, l, KK3_KDA_K), lptr<bf16>(a, l, KK3_KDA_V),
                           lptr<bf16>(a, l, KK3_KDA_OUTPUT_GATE)};
      for (int i = 0; i < 3; ++i) {
        jobs[i].w = wq[i]; jobs[i].rows = g.qdim; jobs[i].out = a.s.qkv + (size_t)i * g.qdim; jobs[i].ldo = 3 * g.qdim;
      }
      jobs[3].w = wq[3]; jobs[3].rows = g.qdim; jobs[3].out = a.s.og; jobs[3].ldo = g.qdim;
      jobs[4].w = lptr<bf16>(a, l, KK3_KDA_FA); jobs[4].rows = g.d; jobs[4].out = a.s.fa; jobs[4].ldo = g.d;
      jobs[5].w = lptr<bf16>(a, l, KK3_KDA_BETA); jobs[5].rows = g.hr; jobs[5].out = a.s.beta; jobs[5].ldo = g.hr;
      for (int i = 0; i < 6; ++i) {
        jobs[i].K = g.h; jobs[i].x = a.s.xa; jobs[i].ldx = g.h; jobs[i].ncols = g.B; jobs[i].epi = EPI_STORE_BF16;
      }
      prepare_jobs(jobs, 6);
      if (KK3_RUN) run_gemv<NT, 1>(a, jobs, 6, 0, gridDim.x, 0);
      KK3_PHASE_END();
      // short conv + gated delta rule (kimi.py:286-299)
      if (KK3_RUN)
        for (int it = blockIdx.x; it < g.B * g.hr; it += gridDim.x) kda_item(a, l, kidx, it / g.hr, it % g.hr, fsm);
      ++kidx;
      KK3_PHASE_END();
    } else {
      // MLA projections q_a, kv_a, output gate (kimi.py:265-266, :282)
      GemvJob jobs[3] = {};
      jobs[0].w = lptr<bf16>(a, l, KK3_MLA_QA); jobs[0].rows = g.qr; jobs[0].out = a.s.qkv; jobs[0].ldo = g.qr;
      jobs[1].w = lptr<bf16>(a, l, KK3_MLA_KA); jobs[1].rows = g.kr + g.rd;
      jobs[1].out = a.s.qkv + (size_t)g.B * g.qr; jobs[1].ldo = g.kr + g.rd;
      jobs[2].w = lptr<bf16>(a, l, KK3_MLA_OUTPUT_GATE); jobs[2].rows = g.hr * g.vd; jobs[2].out = a.s.og;
      jobs[2].ldo = g.hr * g.vd;
      for (int i = 0; i < 3; ++i) {
        jobs[i].K = g.h; jobs[i].x = a.s.xa; jobs[i].ldx = g.h; jobs[i].ncols = g.B; jobs[i].epi = EPI_STORE_BF16;
      }
      prepare_jobs(jobs, 3);
      if (KK3_RUN) run_gemv<NT, 1>(a, jobs, 3, 0, gridDim.x, 0);
      KK3_PHASE_END();
      if (KK3_RUN) phase_mla_rows(a, l, midx, fsm);
      KK3_PHASE_END();
      // q_b (kimi.py:265)
      GemvJob qb = {};
      qb.w = lptr<bf16>(a, l, KK3_MLA_QB); qb.rows = g.hr * (g.nr + g.rd); qb.K = g.qr; qb.x = a.s.mla_qan;
      qb.ldx = g.qr; qb.ncols = g.B; qb.epi = EPI_STORE_BF16; qb.out = a.s.mla_q; qb.ldo = g.hr * (g.nr + g.rd);
      prepare_jobs(&qb, 1);
      if (KK3_RUN) run_gemv<NT, 1>(a, &qb, 1, 0, gridDim.x, 0);
      KK3_PHASE_END();
      // absorbed query (kimi.py:271-272)
      if (KK3_RUN)
        for (int it = blockIdx.x; it < g.hr * 4; it += gridDim.x) mla_absorb_item(a, l, it / 4, it % 4, fsm);
      KK3_PHASE_END();
      // split-K attention over [cache, new token] (kimi.py:274-280)
      if (KK3_RUN) {
        const bool* reset = gptr<bool>(a, KK3_RESET);
        int total = 0;
        for (int b = 0; b < g.B; ++b) total += reset[b] ? 1 : g.mla_chunks;
        for (int it = blockIdx.x; it < total; it += gridDim.x) {
          int b = 0, rem = it;
          for (; b < g.B; ++b) {
            const int n = reset[b] ? 1 : g.mla_chunks;
            if (rem < n) break;
            rem -= n;
          }
          const int T = reset[b] ? 1 : g.ctx + 1;
          const int p0 = rem * g.mla_chunk_len;
          int p1 = p0 + g.mla_chunk_len;
          p1 = p1 < T ? p1 : T;
          mla_attend_item(a, l, midx, b, rem, p0, p1, T, smem);
        }
      }
      KK3_PHASE_END();
      if (KK3_RUN)
        for (int it = blockIdx.x; it < g.B * g.hr; it += gridDim.x) mla_combine_item(a, l, it / g.hr, it % g.hr, fsm);
      ++midx;
      KK3_PHASE_END();
    }
    // o projection -> exchange (kimi.py:283 / :299)
    {
      GemvJob o = {};
      o.w = lptr<bf16>(a, l, KK3_KDA_O); o.rows = g.h; o.K = g.hr * g.vd; o.x = a.s.attn_in; o.ldx = g.hr * g.vd;
      o.ncols = g.B; o.epi = EPI_EXCHANGE; o.ldo = g.h; o.aux_off = a.comm.att_off;
      prepare_jobs(&o, 1);
      if (KK3_RUN) run_gemv<NT, 1>(a, &o, 1, 0, gridDim.x, xi & 1);
      if (g.tp > 1) __threadfence_system();
    }
    const unsigned x_att = xi++;
    KK3_PHASE_END();
    const int nb_after = nb;
    if (KK3_RUN && !phase_mlp_prologue(a, l, nb_after, seq0 + x_att, x_att & 1, fsm)) return;
    KK3_PHASE_END();
    if (l < g.first_dense) {
      // dense FFN (kimi.py:304)
      GemvJob gu = {};
      gu.w = lptr<bf16>(a, l, KK3_DENSE_GATE); gu.w2 = lptr<bf16>(a, l, KK3_DENSE_UP); gu.rows = g.dinter; gu.K = g.h;
      gu.x = a.s.xm; gu.ldx = g.h; gu.ncols = g.B; gu.epi = EPI_SITU; gu.out = a.s.dense_act; gu.ldo = g.dinter;
      prepare_jobs(&gu, 1);
      if (KK3_RUN) run_gemv<NT, 2>(a, &gu, 1, 0, gridDim.x, 0);
      KK3_PHASE_END();
      GemvJob dn = {};
      dn.w = lptr<bf16>(a, l, KK3_DENSE_DOWN); dn.rows = g.h; dn.K = g.dinter; dn.x = a.s.dense_act; dn.ldx = g.dinter;
      dn.ncols = g.B; dn.epi = EPI_EXCHANGE; dn.ldo = g.h; dn.aux_off = a.comm.att_off;
      prepare_jobs(&dn, 1);
      if (KK3_RUN) run_gemv<NT, 1>(a, &dn, 1, 0, gridDim.x, xi & 1);
      if (g.tp > 1) __threadfence_system();
      pending = PEND_DENSE;
      pend_signal = true;
      pend_x = xi++;
      KK3_PHASE_END();
    } else {
      // router, latent down (pass 0) and shared gate/up (pass 1) (kimi.py:308, :317, :326)
      GemvJob j0[2] = {};
      j0[0].w = lptr<bf16>(a, l, KK3_MOE_ROUTER); j0[0].rows = g.E; j0[0].epi = EPI_SIGMOID_F32; j0[0].out = a.s.scores;
      j0[0].ldo = g.E;
      j0[1].w = lptr<bf16>(a, l, KK3_MOE_LATENT_DOWN); j0[1].rows = g.lh; j0[1].epi = EPI_LATENT; j0[1].out = a.s.latent;
      j0[1].out2 = a.s.latent_p; j0[1].ldo = g.lh;
      for (int i = 0; i < 2; ++i) {
        j0[i].K = g.h; j0[i].x = a.s.xm; j0[i].ldx = g.h; j0[i].ncols = g.B;
      }
      prepare_jobs(j0, 2);
      if (KK3_RUN) run_gemv<NT, 1>(a, j0, 2, 0, gridDim.x, 0, 0);
      GemvJob j1 = {};
      j1.w = lptr<bf16>(a, l, KK3_MOE_SHARED_GATE); j1.w2 = lptr<bf16>(a, l, KK3_MOE_SHARED_UP); j1.rows = g.sinter;
      j1.K = g.h; j1.x = a.s.xm; j1.ldx = g.h; j1.ncols = g.B; j1.epi = EPI_SITU; j1.out = a.s.shared_act; j1.ldo = g.sinter;
      prepare_jobs(&j1, 1);
      if (KK3_RUN) run_gemv<NT, 2>(a, &j1, 1, 0, gridDim.x, 0, 1);
      KK3_PHASE_END();
      // routing on CTA 0 while the other CTAs run the shared-expert down projection (kimi.py:309-316, :326)
      const unsigned x_moe = xi++;
      if (!KK3_RUN) {
      } else if (blockIdx.x == 0) {
        route_all(a, l, l - g.first_dense, smem);
      } else {
        GemvJob sd = {};
        sd.w = lptr<bf16>(a, l, KK3_MOE_SHARED_DOWN); sd.rows = g.h; sd.K = g.sinter; sd.x = a.s.shared_act;
        sd.ldx = g.sinter; sd.ncols = g.B; sd.epi = EPI_EXCHANGE; sd.ldo = g.h; sd.aux_off = a.comm.shd_off;
        prepare_jobs(&sd, 1);
        run_gemv<NT, 1>(a, &sd, 1, 1, gridDim.x, x_moe & 1);
        if (g.tp > 1) __threadfence_system();
      }
      KK3_PHASE_END();
      // routed experts (kimi.py:317-323)
      {
        ExpertPhase ph;
        ph.codes[0] = lptr<uint8_t>(a, l, KK3_MOE_GATE_BLOCKS);
        ph.codes[1] = lptr<uint8_t>(a, l, KK3_MOE_UP_BLOCKS);
        ph.scales[0] = lptr<uint8_t>(a, l, KK3_MOE_GATE_SCALES);
        ph.scales[1] = lptr<uint8_t>(a, l, KK3_MOE_UP_SCALES);
        ph.rows = g.inter; ph.K = g.lh; ph.tiles = g.inter / 16; ph.ksteps = g.lh / 64;
        ph.expert_codes = (long long)g.inter * g.lh / 2; ph.expert_scales = (long long)g.inter * g.lh / 32;
        if (KK3_RUN) run_experts<2>(a, ph);
      }
      KK3_PHASE_END();
      {
        ExpertPhase ph;
        ph.codes[0] = ph.codes[1] = lptr<uint8_t>(a, l, KK3_MOE_DOWN_BLOCKS);
        ph.scales[0] = ph.scales[1] = lptr<uint8_t>(a, l, KK3_MOE_DOWN_SCALES);
        ph.rows = g.lh; ph.K = g.inter; ph.tiles = g.lh / 16; ph.ksteps = g.inter / 64;
        ph.expert_codes = (long long)g.lh * g.inter / 2; ph.expert_scales = (long long)g.lh * g.inter / 32;
        if (KK3_RUN) run_experts<1>(a, ph);
      }
      KK3_PHASE_END();
      if (KK3_RUN && !phase_moe_combine(a, l, seq0 + x_moe, x_moe & 1, fsm)) return;
      KK3_PHASE_END();
      // latent up + shared + residual (kimi.py:325-329)
      GemvJob up = {};
      up.w = lptr<bf16>(a, l, KK3_MOE_LATENT_UP); up.rows = g.h; up.K = g.lh; up.x = a.s.x3; up.ldx = g.lh;
      up.ncols = g.B; up.epi = EPI_ROUTED; up.out = a.s.prefix; up.aux = a.s.shared_red; up.ldo = g.h;
      prepare_jobs(&up, 1);
      if (KK3_RUN) run_gemv<NT, 1>(a, &up, 1, 0, gridDim.x, 0);
      KK3_PHASE_END();
    }
  }
  // head (kimi.py:330-334)
  if (pending != PEND_NONE) {
    // the last layer was dense: fold its exchange into prefix first
    if (KK3_RUN && !phase_fold_pending(a, pending, pend_signal, seq0 + pend_x, pend_x & 1)) return;
    KK3_PHASE_END();
  }
  if (KK3_RUN) phase_head_prologue(a, nb, fsm);
  KK3_PHASE_END();
  {
    GemvJob hd = {};
    hd.w = gptr<bf16>(a, KK3_LM_HEAD); hd.rows = g.V; hd.K = g.h; hd.x = a.s.xa; hd.ldx = g.h; hd.ncols = g.B;
    hd.epi = EPI_LOGITS; hd.out = gout<float>(a, KK3_OUT_LOGITS); hd.ldo = g.V; hd.aux = a.s.argmax_key;
    hd.aux_off = (long long)g.rank * g.V;
    prepare_jobs(&hd, 1);
    if (KK3_RUN) run_gemv<NT, 1>(a, &hd, 1, 0, gridDim.x, 0);
  }
  KK3_PHASE_END();
  const unsigned x_key = xi++;
  if (KK3_RUN && !phase_argmax(a, seq0 + x_key, x_key & 1)) return;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (phase + 1 <= kMaxPhases) a.s.phase_ts[phase + 1] = globaltimer();
    *a.s.phase_count = phase + 1;
  }
#undef KK3_PHASE_END
#undef KK3_RUN
}

}  // namespace kk3

