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
#include "kk3_tc_gemv.cuh"

namespace kk3 {

KK3_DEV bool layer_is_mla(const Geo& g, int l) { return ((l + 1) % 4 == 0) || (l == g.L - 1); }

enum Pending : int { PEND_NONE = 0, PEND_EMBED, PEND_DENSE };

// ---- row phases ------------------------------------------------------------------------------------

KK3_FN void phase_embed(const StepArgs& a, unsigned seq, int parity, float* fsm) {
  const Geo& g = a.g;
  const long long* tok = gptr<long long>(a, KK3_TOKEN);
  const bf16* emb = gptr<bf16>(a, KK3_EMBED);
  long long* out_ids = gout<long long>(a, KK3_OUT_EXPERT_IDS);
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    const long long t = tok[b] - (long long)g.rank * g.V;
    const bool mine = t >= 0 && t < g.V;
    const bf16* row = emb + (size_t)(mine ? t : 0) * g.h;
    const bf16 zero = f2bf(0.0f);
    if (g.tp == 1) {
      #pragma unroll 1
      for (int e = threadIdx.x; e < g.h; e += kThreads) a.s.prefix[(size_t)b * g.h + e] = mine ? row[e] : zero;
    } else {
      // 16-byte pieces of the row into every rank's att region (layout xch_index)
      #pragma unroll 1
      for (int c = threadIdx.x; c < g.h / 8; c += kThreads) {
        const uint4 v = mine ? *reinterpret_cast<const uint4*>(row + (size_t)c * 8) : make_uint4(0, 0, 0, 0);
        const size_t e = xch_index(g, g.rank, b, c * 8, g.h);
        #pragma unroll 1
        for (int dst = xdst_lo(a); dst < xdst_hi(a); ++dst)
          *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.comm.base[dst] + a.comm.data_off[parity] + a.comm.att_off) + e) = v;
      }
      xch_signal_row(a, b, seq);
    }
    // dense layers report -1 expert ids (kimi.py:305)
    #pragma unroll 1
    for (int l = 0; l < g.first_dense && l < g.L; ++l)
      #pragma unroll 1
      for (int j = threadIdx.x; j < g.K; j += kThreads) out_ids[((size_t)l * g.B + b) * g.K + j] = -1;
  }
  (void)fsm;
}

// load this thread's chunks of prefix row b, folding a pending exchange in first (embedding: assign;
// dense FFN / attention: add, or assign right after a block push), and write the result back
KK3_DEV void load_prefix(const StepArgs& a, int b, int fold, bool assign, int parity, uint4 (&pre)[kRowChunks]) {
  const Geo& g = a.g;
  const int nvec = g.h / 8;
  bf16* row = a.s.prefix + (size_t)b * g.h;
#pragma unroll
  for (int q = 0; q < kRowChunks; ++q) {
    const int c = threadIdx.x + q * kThreads;
    pre[q] = make_uint4(0, 0, 0, 0);
    if (c >= nvec) continue;
    if (!fold) {
      pre[q] = ld_act16(row + c * 8);
      continue;
    }
    float x[8], old[8];
    xch_sum8(a, parity, a.comm.att_off, b, g.h, c, x);
    if (!assign) {
      unpack8(ld_act16(row + c * 8), old);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = round_bf(old[e] + x[e]);
    }
    pre[q] = pack8(x);
    *reinterpret_cast<uint4*>(row + c * 8) = pre[q];
  }
}

KK3_DEV void store_row(bf16* dst, const uint4 (&v)[kRowChunks], int nvec) {
#pragma unroll
  for (int q = 0; q < kRowChunks; ++q) {
    const int c = threadIdx.x + q * kThreads;
    if (c < nvec) *reinterpret_cast<uint4*>(dst + c * 8) = v[q];
  }
}

// finish a pending exchange into prefix (embedding: assign; dense FFN: add), then the attention prologue
KK3_FN bool phase_attn_prologue(const StepArgs& a, int layer, int nb, int pending, bool need_signal, unsigned seq,
                                 int parity, float* fsm, int ph = -1) {
  const Geo& g = a.g;
  // push transport: the dense FFN's partial is pushed here (the embedding rows were stored directly)
  const bool push = a.comm_mode == kCommPush && g.tp > 1 && pending == PEND_DENSE;
  if (push) xch_push(a, parity, a.comm.att_off, (long long)g.h * g.bp * 2, seq);
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (b == 0 && threadIdx.x == 0) sub_stamp(a, ph, 0);
    const bool fold = pending != PEND_NONE && !(g.tp == 1 && pending == PEND_EMBED);
    if (push) {
      if (!xch_wait_push(a, seq)) return false;
    } else if (pending != PEND_NONE && g.tp > 1) {
      if (need_signal) xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
    }
    uint4 pre[kRowChunks];
    load_prefix(a, b, fold, pending == PEND_EMBED, parity, pre);
    mix_and_norm_regs(a, b, nb, pre, gptr<bf16>(a, KK3_ATTENTION_RES_NORM) + (size_t)layer * g.h,
                      gptr<bf16>(a, KK3_ATTENTION_RES_PROJ) + (size_t)layer * g.h,
                      gptr<bf16>(a, KK3_LN1) + (size_t)layer * g.h, 1e-5f, a.s.xa + (size_t)b * g.h, fsm, ph);
    if (b == 0 && threadIdx.x == 0) sub_stamp(a, ph, 6);
    if (layer % g.bs == 0) store_row(a.s.blocks + ((size_t)nb * g.B + b) * g.h, pre, g.h / 8);
    __syncthreads();
  }
  return true;
}

// fold a pending exchange into prefix without a following norm (only when the last layer is dense)
KK3_FN bool phase_fold_pending(const StepArgs& a, int pending, bool need_signal, unsigned seq, int parity) {
  const Geo& g = a.g;
  const bool push = a.comm_mode == kCommPush && g.tp > 1 && pending == PEND_DENSE;
  if (push) xch_push(a, parity, a.comm.att_off, (long long)g.h * g.bp * 2, seq);
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (push) {
      if (!xch_wait_push(a, seq)) return false;
    } else if (g.tp > 1) {
      if (need_signal) xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
    }
    uint4 pre[kRowChunks];
    load_prefix(a, b, 1, pending == PEND_EMBED, parity, pre);
    __syncthreads();
  }
  return true;
}

// attention exchange -> prefix (assign right after a block push, else add), then the MLP prologue
KK3_FN bool phase_mlp_prologue(const StepArgs& a, int layer, int nb_after, unsigned seq, int parity, float* fsm) {
  const Geo& g = a.g;
  const bool push = a.comm_mode == kCommPush && g.tp > 1;
  if (push) xch_push(a, parity, a.comm.att_off, (long long)g.h * g.bp * 2, seq);
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (push) {
      if (!xch_wait_push(a, seq)) return false;
    } else if (g.tp > 1) {
      xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
    }
    uint4 pre[kRowChunks];
    load_prefix(a, b, 1, (layer % g.bs) == 0, parity, pre);
    mix_and_norm_regs(a, b, nb_after, pre, gptr<bf16>(a, KK3_MLP_RES_NORM) + (size_t)layer * g.h,
                      gptr<bf16>(a, KK3_MLP_RES_PROJ) + (size_t)layer * g.h, gptr<bf16>(a, KK3_LN2) + (size_t)layer * g.h,
                      1e-5f, a.s.xm + (size_t)b * g.h, fsm);
    __syncthreads();
  }
  return true;
}

// MLA row prologue: q_a norm, latent norm (-> kv_write), rope part (-> pe_write)  (kimi.py:265-270)
KK3_FN void phase_mla_rows(const StepArgs& a, int layer, int midx, float* fsm) {
  const Geo& g = a.g;
  const bf16* qa = a.s.qkv;
  const bf16* ka = a.s.qkv + (size_t)g.B * g.qr;
  bf16* kvw = gout<bf16>(a, KK3_OUT_KV_WRITE) + (size_t)midx * g.B * g.kr;
  bf16* pew = gout<bf16>(a, KK3_OUT_PE_WRITE) + (size_t)midx * g.B * g.rd;
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    rms_row(qa + (size_t)b * g.qr, lptr<bf16>(a, layer, KK3_MLA_QN), g.qr, 1e-6f, a.s.mla_qan + (size_t)b * g.qr, fsm);
    rms_row(ka + (size_t)b * (g.kr + g.rd), lptr<bf16>(a, layer, KK3_MLA_KN), g.kr, 1e-6f, kvw + (size_t)b * g.kr, fsm);
    #pragma unroll 1
    for (int e = threadIdx.x; e < g.rd; e += kThreads) pew[(size_t)b * g.rd + e] = ka[(size_t)b * (g.kr + g.rd) + g.kr + e];
    __syncthreads();
    if (a.lengths != nullptr) {
      // append mode: the row's new latent and rope entries also go into its cache at position `length` (0 after
      // a reset); the attention phases read only positions below it, and the new token from kv_write/pe_write
      const bool rst = reinterpret_cast<const bool*>(a.ptr[KK3_RESET])[b];
      const long long n = rst ? 0 : a.lengths[b];
      if (n < 0 || n >= g.ctx) {
        if (threadIdx.x == 0) set_error(a, kErrDevice);   // the cache is full (or the length is invalid)
      } else {
        bf16* kvc = const_cast<bf16*>(lptr<bf16>(a, layer, KK3_MLA_KV_CACHE)) + ((size_t)b * g.ctx + n) * g.kr;
        bf16* pec = const_cast<bf16*>(lptr<bf16>(a, layer, KK3_MLA_PE_CACHE)) + ((size_t)b * g.ctx + n) * g.rd;
        #pragma unroll 1
        for (int e = threadIdx.x; e < g.kr; e += kThreads) kvc[e] = kvw[(size_t)b * g.kr + e];
        #pragma unroll 1
        for (int e = threadIdx.x; e < g.rd; e += kThreads) pec[e] = pew[(size_t)b * g.rd + e];
      }
      __syncthreads();
    }
  }
}

// MoE combine: expert_sum (slot order = ascending expert id, kimi.py:319-323), TP sum (:324),
// latent_norm (:325) -> x3; shared-expert TP sum (:326) -> shared_red.
// `part`: kCombineAll runs it whole (the in-kernel exchange waits for the peers' slots in the middle). With the
// host transport it is two phases: kCombineWrite ends after this rank's slot is written (the launch ends there
// and the host all-reduces the slots), kCombineRead starts from the reduced slot.
constexpr int kCombineAll = 0, kCombineWrite = 1, kCombineRead = 2;
KK3_FN bool phase_moe_combine_rows(const StepArgs& a, int layer, unsigned seq, int parity, float* fsm, int part) {
  const Geo& g = a.g;
  float* red = fsm;
  const int nvec = g.lh / 8, hvec = g.h / 8;
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    const float* w = a.s.route_w + (size_t)b * g.K;
    float tot[kRowChunks][8];
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) {
      const int c = threadIdx.x + q * kThreads;
#pragma unroll
      for (int e = 0; e < 8; ++e) tot[q][e] = 0.0f;
      if (c >= nvec || part == kCombineRead) continue;
      // 8 slots' loads in flight at a time (L2), summed in slot order
      const uint4* slot0 = reinterpret_cast<const uint4*>(a.s.out_slot + (size_t)b * g.K * g.lh) + c;
      #pragma unroll 1
      for (int j0 = 0; j0 < g.K; j0 += 8) {
        uint4 v[8];
        float wj[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const bool live = j0 + u < g.K;
          v[u] = live ? __ldcg(slot0 + (size_t)(j0 + u) * nvec) : make_uint4(0, 0, 0, 0);
          wj[u] = live ? __ldcg(w + j0 + u) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (j0 + u >= g.K) break;
          float f[8];
          unpack8(v[u], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) tot[q][e] += f[e] * wj[u];
        }
      }
      float* es = a.s.expert_sum + (size_t)b * g.lh + c * 8;
      *reinterpret_cast<float4*>(es) = make_float4(tot[q][0], tot[q][1], tot[q][2], tot[q][3]);
      *reinterpret_cast<float4*>(es + 4) = make_float4(tot[q][4], tot[q][5], tot[q][6], tot[q][7]);
    }
    if (g.tp > 1) {
      const size_t off = ((size_t)g.rank * g.B + b) * g.lh;
      if (part != kCombineRead) {
        #pragma unroll 1
        for (int dst = xdst_lo(a); dst < xdst_hi(a); ++dst) {
          float* reg = reinterpret_cast<float*>(a.comm.base[dst] + a.comm.data_off[parity] + a.comm.exp_off) + off;
#pragma unroll
          for (int q = 0; q < kRowChunks; ++q) {
            const int c = threadIdx.x + q * kThreads;
            if (c >= nvec) continue;
            *reinterpret_cast<float4*>(reg + c * 8) = make_float4(tot[q][0], tot[q][1], tot[q][2], tot[q][3]);
            *reinterpret_cast<float4*>(reg + c * 8 + 4) = make_float4(tot[q][4], tot[q][5], tot[q][6], tot[q][7]);
          }
        }
        if (part == kCombineWrite) continue;   // the host all-reduces the slots before kCombineRead
        xch_signal_row(a, b, seq);
        if (!xch_wait_row(a, b, seq)) return false;
      }
      const float* reg = xlocal<float>(a, parity, a.comm.exp_off);
      // peer stores: every rank's slot, summed in rank order; host transport: the all-reduced own slot
      const int lo = a.comm_mode == kCommHost ? g.rank : 0, hi = a.comm_mode == kCommHost ? g.rank + 1 : g.tp;
#pragma unroll
      for (int q = 0; q < kRowChunks; ++q) {
        const int c = threadIdx.x + q * kThreads;
        if (c >= nvec) continue;
#pragma unroll
        for (int e = 0; e < 8; ++e) tot[q][e] = 0.0f;
        #pragma unroll 1
        for (int src = lo; src < hi; ++src) {
          const float* r = reg + ((size_t)src * g.B + b) * g.lh + c * 8;
          const float4 v0 = *reinterpret_cast<const float4*>(r), v1 = *reinterpret_cast<const float4*>(r + 4);
          tot[q][0] += v0.x; tot[q][1] += v0.y; tot[q][2] += v0.z; tot[q][3] += v0.w;
          tot[q][4] += v1.x; tot[q][5] += v1.y; tot[q][6] += v1.z; tot[q][7] += v1.w;
        }
      }
    }
    // x3 = rms(bf16(total), latent_norm)
    float ss[1] = {0.0f};
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        tot[q][e] = round_bf(tot[q][e]);
        ss[0] += tot[q][e] * tot[q][e];
      }
    block_sums<1>(ss, red);
    const float rs = rsqrtf(ss[0] / (float)g.lh + 1e-5f);
    const bf16* ln = lptr<bf16>(a, layer, KK3_MOE_LATENT_NORM);
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) {
      const int c = threadIdx.x + q * kThreads;
      if (c >= nvec) continue;
      float wf[8], o[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(ln) + c), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = round_bf(round_bf(tot[q][e] * rs) * wf[e]);
      *reinterpret_cast<uint4*>(a.s.x3 + (size_t)b * g.lh + c * 8) = pack8(o);
    }
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) {
      const int c = threadIdx.x + q * kThreads;
      if (c >= hvec) continue;
      float x[8];
      xch_sum8(a, parity, a.comm.shd_off, b, g.h, c, x);
      *reinterpret_cast<uint4*>(a.s.shared_red + (size_t)b * g.h + c * 8) = pack8(x);
    }
    __syncthreads();
  }
  return true;
}

// Weighted sum of the K pair outputs of row b, channels 8v .. 8v + 7, in slot order (kimi.py:320-323: each
// pair's output times its routing weight, accumulated in FP32)
KK3_DEV void routed_sum8(const StepArgs& a, int b, int v, float (&tot)[8]) {
  const Geo& g = a.g;
  const int nvec = g.lh / 8;
  const float* w = a.s.route_w + (size_t)b * g.K;
  const uint4* slot0 = reinterpret_cast<const uint4*>(a.s.out_slot + (size_t)b * g.K * g.lh) + v;
#pragma unroll
  for (int e = 0; e < 8; ++e) tot[e] = 0.0f;
  #pragma unroll 1
  for (int j0 = 0; j0 < g.K; j0 += 8) {
    uint4 x[8];
    float wj[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const bool live = j0 + u < g.K;
      x[u] = live ? __ldcg(slot0 + (size_t)(j0 + u) * nvec) : make_uint4(0, 0, 0, 0);
      wj[u] = live ? __ldcg(w + j0 + u) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (j0 + u >= g.K) break;
      float f[8];
      unpack8(x[u], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) tot[e] += f[e] * wj[u];
    }
  }
}

// MoE combine with the in-kernel transports at TP > 1. The routed sums are computed in B x Q chunk items (Q =
// min(G / B, lh / 32) per row), item i on CTA i, and every item stores its FP32 chunk into the exp slot of this
// rank in every rank's buffer (own included); under the push transport every CTA also pushes its share of the
// shared expert's partial. Then every CTA raises flag [rank][cta] = seq in every buffer, so each SM sends a few
// KB instead of the row CTAs sending whole rows. The row CTAs wait for all flags and finish as the row path does:
// FP32 sum of the tp slots in rank order (kimi.py:343-347), latent norm, shared-expert sum.
KK3_FN bool phase_moe_combine_chunked(const StepArgs& a, int layer, unsigned seq, int parity, float* fsm) {
  const Geo& g = a.g;
  float* red = fsm;
  const int nvec = g.lh / 8, hvec = g.h / 8;
  if (a.comm_mode == kCommPush) xch_push_stores(a, parity, a.comm.shd_off, (long long)g.h * g.bp * 2);
  int Q = (int)gridDim.x / g.B;
  Q = Q < nvec / 4 ? Q : nvec / 4;
  Q = Q < 1 ? 1 : Q;
  if ((int)blockIdx.x < g.B * Q) {
    const int b = blockIdx.x / Q, q = blockIdx.x - b * Q;
    const int v0 = nvec * q / Q, v1 = nvec * (q + 1) / Q;
    const size_t off = ((size_t)g.rank * g.B + b) * g.lh;
    for (int v = v0 + threadIdx.x; v < v1; v += kThreads) {
      float tot[8];
      routed_sum8(a, b, v, tot);
      const float4 lo = make_float4(tot[0], tot[1], tot[2], tot[3]), hi = make_float4(tot[4], tot[5], tot[6], tot[7]);
      #pragma unroll 1
      for (int dst = 0; dst < g.tp; ++dst) {
        float* reg = reinterpret_cast<float*>(a.comm.base[dst] + a.comm.data_off[parity] + a.comm.exp_off) + off + v * 8;
        *reinterpret_cast<float4*>(reg) = lo;
        *reinterpret_cast<float4*>(reg + 4) = hi;
      }
    }
  }
  xch_push_flags(a, seq, false);
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (!xch_wait_push(a, seq, true)) return false;
    const float* reg = xlocal<float>(a, parity, a.comm.exp_off);
    float tot[kRowChunks][8];
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) {
      const int c = threadIdx.x + q * kThreads;
#pragma unroll
      for (int e = 0; e < 8; ++e) tot[q][e] = 0.0f;
      if (c >= nvec) continue;
      #pragma unroll 1
      for (int src = 0; src < g.tp; ++src) {
        const float* r = reg + ((size_t)src * g.B + b) * g.lh + c * 8;
        const float4 v0 = __ldcg(reinterpret_cast<const float4*>(r)), v1 = __ldcg(reinterpret_cast<const float4*>(r + 4));
        tot[q][0] += v0.x; tot[q][1] += v0.y; tot[q][2] += v0.z; tot[q][3] += v0.w;
        tot[q][4] += v1.x; tot[q][5] += v1.y; tot[q][6] += v1.z; tot[q][7] += v1.w;
      }
    }
    // x3 = rms(bf16(total), latent_norm)
    float ss[1] = {0.0f};
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        tot[q][e] = round_bf(tot[q][e]);
        ss[0] += tot[q][e] * tot[q][e];
      }
    block_sums<1>(ss, red);
    const float rs = rsqrtf(ss[0] / (float)g.lh + 1e-5f);
    const bf16* ln = lptr<bf16>(a, layer, KK3_MOE_LATENT_NORM);
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) {
      const int c = threadIdx.x + q * kThreads;
      if (c >= nvec) continue;
      float wf[8], o[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(ln) + c), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = round_bf(round_bf(tot[q][e] * rs) * wf[e]);
      *reinterpret_cast<uint4*>(a.s.x3 + (size_t)b * g.lh + c * 8) = pack8(o);
    }
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) {
      const int c = threadIdx.x + q * kThreads;
      if (c >= hvec) continue;
      float x[8];
      xch_sum8(a, parity, a.comm.shd_off, b, g.h, c, x);
      *reinterpret_cast<uint4*>(a.s.shared_red + (size_t)b * g.h + c * 8) = pack8(x);
    }
    __syncthreads();
  }
  return true;
}

KK3_FN bool phase_moe_combine(const StepArgs& a, int layer, unsigned seq, int parity, float* fsm, int part) {
  if (a.g.tp > 1 && a.comm_mode != kCommHost) return phase_moe_combine_chunked(a, layer, seq, parity, fsm);
  return phase_moe_combine_rows(a, layer, seq, parity, fsm, part);
}

KK3_FN void phase_head_prologue(const StepArgs& a, int nb, float* fsm) {
  const Geo& g = a.g;
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    uint4 pre[kRowChunks];
    load_prefix(a, b, 0, false, 0, pre);
    mix_and_norm_regs(a, b, nb, pre, gptr<bf16>(a, KK3_OUTPUT_RES_NORM), gptr<bf16>(a, KK3_OUTPUT_RES_PROJ),
                      gptr<bf16>(a, KK3_FNORM), 1e-5f, a.s.xa + (size_t)b * g.h, fsm);
    if (threadIdx.x == 0) a.s.argmax_key[b] = 0ull;
    __syncthreads();
  }
}

// Greedy token (kimi.py:218-227): the largest (value, lowest index) key over the ranks. `part` as in
// phase_moe_combine: with the host transport, kCombineWrite stores this rank's key and the launch ends (the host
// all-gathers the keys), kCombineRead takes the maximum over the gathered slots.
KK3_FN bool phase_argmax(const StepArgs& a, unsigned seq, int parity, int part) {
  const Geo& g = a.g;
  long long* next = gout<long long>(a, KK3_OUT_NEXT_TOKEN);
  long long* len = gout<long long>(a, KK3_OUT_CACHE_LENGTH);
  const bool* reset = gptr<bool>(a, KK3_RESET);
  __shared__ unsigned long long best;
  #pragma unroll 1
  for (int b = blockIdx.x; b < g.B; b += gridDim.x) {
    if (threadIdx.x == 0) best = *reinterpret_cast<volatile unsigned long long*>(a.s.argmax_key + b);
    __syncthreads();
    if (g.tp > 1) {
      const size_t off = (size_t)g.rank * g.B + b;
      if ((int)threadIdx.x < g.tp && part != kCombineRead &&
          ((int)threadIdx.x >= xdst_lo(a) && (int)threadIdx.x < xdst_hi(a))) {
        unsigned long long* reg =
            reinterpret_cast<unsigned long long*>(a.comm.base[threadIdx.x] + a.comm.data_off[parity] + a.comm.key_off);
        reg[off] = best;
      }
      if (part == kCombineWrite) {
        __syncthreads();
        continue;
      }
      xch_signal_row(a, b, seq);
      if (!xch_wait_row(a, b, seq)) return false;
      if (threadIdx.x == 0) {
        const unsigned long long* reg = xlocal<unsigned long long>(a, parity, a.comm.key_off);
        unsigned long long m = 0ull;
        #pragma unroll 1
        for (int src = 0; src < g.tp; ++src) {
          const unsigned long long k = reg[(size_t)src * g.B + b];
          m = k > m ? k : m;
        }
        best = m;
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      // an error raised earlier in the step (a full append cache, for one) is visible here through the grid
      // barriers since: the step's outputs are then marked invalid instead of written
      const bool bad = failed(a);
      next[b] = bad ? -1 : (long long)(0xffffffffu - (unsigned)(best & 0xffffffffull));
      len[b] = bad ? 0 : (reset[b] ? 1 : (long long)(a.lengths ? mla_row_len(a, b) : g.ctx) + 1);
    }
    __syncthreads();
  }
  return true;
}

// The row phases read a few per-layer vectors once each, at the head of latency-bound chains. The phase
// before each of them asks for those vectors in L2 (three bulk prefetches from the last CTA), so the row
// phase finds them there instead of in HBM.
KK3_DEV void prefetch_vectors(const void* v0, const void* v1, const void* v2, int bytes) {
  if (blockIdx.x != gridDim.x - 1 || threadIdx.x >= 3) return;
  const void* v = threadIdx.x == 0 ? v0 : (threadIdx.x == 1 ? v1 : v2);
  const unsigned n = (unsigned)bytes & ~15u;
  if (v && (reinterpret_cast<uintptr_t>(v) & 15u) == 0 && n >= 16) prefetch_l2(v, n);
}
// attention (which = 0) or MLP (1) prologue vectors of layer l, the head's (l = L), or the latent norm (2)
KK3_DEV void prefetch_row_inputs(const StepArgs& a, int which, int l) {
  const Geo& g = a.g;
  if (which == 2) {
    prefetch_vectors(lptr<bf16>(a, l, KK3_MOE_LATENT_NORM), nullptr, nullptr, g.lh * 2);
  } else if (l >= g.L) {
    prefetch_vectors(gptr<bf16>(a, KK3_FNORM), gptr<bf16>(a, KK3_OUTPUT_RES_NORM), gptr<bf16>(a, KK3_OUTPUT_RES_PROJ),
                     g.h * 2);
  } else {
    const size_t o = (size_t)l * g.h;
    prefetch_vectors(gptr<bf16>(a, which ? KK3_MLP_RES_NORM : KK3_ATTENTION_RES_NORM) + o,
                     gptr<bf16>(a, which ? KK3_MLP_RES_PROJ : KK3_ATTENTION_RES_PROJ) + o,
                     gptr<bf16>(a, which ? KK3_LN2 : KK3_LN1) + o, g.h * 2);
  }
}

// One BF16 GEMV pass over all CTAs: the tcgen05 engine for the batch classes above 16 rows (NT >= 4), the
// warp-level mma.sync engine below (and for every batch when the context asks for it). False when a bounded
// wait of the tcgen05 engine gave up.
template <int NT>
KK3_DEV bool gemv_pass(const StepArgs& a, const GemvJob* jobs, int njobs, int parity, int bank = 0, int ph = -1) {
  if constexpr (NT >= 4) {
    if (a.gemv_engine == kGemvAuto) return run_gemv_tc<NT>(a, jobs, njobs, parity, bank);
  }
  run_gemv<NT, 1>(a, jobs, njobs, 0, gridDim.x, parity, bank, ph);
  return true;
}

// the MXFP4 down projection runs as row pairs (run_experts<2, true>) when its 32-row tiles and scale layout fit
KK3_DEV bool down_row_pairs(const Geo& g) {
  return g.lh % 32 == 0 && (g.inter % 512 == 0 || g.inter <= 512);
}

// ---- job lists of the GEMV phases (built identically by every thread) ---------------------------------

KK3_DEV void job_init(GemvJob& j, const bf16* w, int rows, int K, const bf16* x, int ldx, int ncols, int epi, void* out,
                      int ldo) {
  j = GemvJob{};
  j.w = w; j.rows = rows; j.K = K; j.x = x; j.ldx = ldx; j.ncols = ncols; j.epi = epi; j.out = out; j.ldo = ldo;
}

// L2 lookahead (prefetch_jobs) is issued only from phases that stream HBM themselves (KDA, MLA combine):
// in the latency-bound row phases the bulk prefetch traffic queued ahead of their few dependent loads.

// attention input projections: KDA q,k,v,g,f_a,beta (kimi.py:285, :290-291, :298) or MLA q_a, kv_a, g (:265-266, :282)
KK3_DEV int attn_proj_jobs(const StepArgs& a, int l, bool mla, GemvJob* jobs) {
  const Geo& g = a.g;
  if (!mla) {
    const int slots[4] = {KK3_KDA_Q, KK3_KDA_K, KK3_KDA_V, KK3_KDA_OUTPUT_GATE};
    for (int i = 0; i < 3; ++i)
      job_init(jobs[i], lptr<bf16>(a, l, slots[i]), g.qdim, g.h, a.s.xa, g.h, g.B, EPI_STORE_BF16,
               a.s.qkv + (size_t)i * g.qdim, 3 * g.qdim);
    job_init(jobs[3], lptr<bf16>(a, l, slots[3]), g.qdim, g.h, a.s.xa, g.h, g.B, EPI_STORE_BF16, a.s.og, g.qdim);
    job_init(jobs[4], lptr<bf16>(a, l, KK3_KDA_FA), g.d, g.h, a.s.xa, g.h, g.B, EPI_STORE_BF16, a.s.fa, g.d);
    job_init(jobs[5], lptr<bf16>(a, l, KK3_KDA_BETA), g.hr, g.h, a.s.xa, g.h, g.B, EPI_STORE_BF16, a.s.beta, g.hr);
    prepare_jobs(jobs, 6);
    return 6;
  }
  job_init(jobs[0], lptr<bf16>(a, l, KK3_MLA_QA), g.qr, g.h, a.s.xa, g.h, g.B, EPI_STORE_BF16, a.s.qkv, g.qr);
  job_init(jobs[1], lptr<bf16>(a, l, KK3_MLA_KA), g.kr + g.rd, g.h, a.s.xa, g.h, g.B, EPI_STORE_BF16,
           a.s.qkv + (size_t)g.B * g.qr, g.kr + g.rd);
  job_init(jobs[2], lptr<bf16>(a, l, KK3_MLA_OUTPUT_GATE), g.hr * g.vd, g.h, a.s.xa, g.h, g.B, EPI_STORE_BF16, a.s.og,
           g.hr * g.vd);
  prepare_jobs(jobs, 3);
  return 3;
}

// o projection -> exchange (kimi.py:283 / :299)
KK3_DEV void o_job(const StepArgs& a, int l, GemvJob& j) {
  const Geo& g = a.g;
  job_init(j, lptr<bf16>(a, l, KK3_KDA_O), g.h, g.hr * g.vd, a.s.attn_in, g.hr * g.vd, g.B, EPI_EXCHANGE, nullptr, g.h);
  j.aux_off = a.comm.att_off;
  prepare_jobs(&j, 1);
}

KK3_DEV void situ_pair(const StepArgs& a, GemvJob* jobs, const bf16* gate, const bf16* up, int rows, bf16* out) {
  const Geo& g = a.g;
  job_init(jobs[0], gate, rows, g.h, a.s.xm, g.h, g.B, EPI_SITU_GATE, out, rows);
  job_init(jobs[1], up, rows, g.h, a.s.xm, g.h, g.B, EPI_SITU_UP, out, rows);
  for (int i = 0; i < 2; ++i) {
    jobs[i].aux = a.s.situ_buf;
    jobs[i].out2 = a.s.situ_cnt;
  }
}

// MLP input in one pass of single-matrix jobs: dense gate and up (kimi.py:304), or router, latent down and the
// shared expert's gate and up (:308, :317, :326); gate/up tiles meet in the situ epilogue
KK3_DEV int mlp_in_jobs(const StepArgs& a, int l, GemvJob* jobs) {
  const Geo& g = a.g;
  if (l < g.first_dense) {
    situ_pair(a, jobs, lptr<bf16>(a, l, KK3_DENSE_GATE), lptr<bf16>(a, l, KK3_DENSE_UP), g.dinter, a.s.dense_act);
    prepare_jobs(jobs, 2);
    return 2;
  }
  job_init(jobs[0], lptr<bf16>(a, l, KK3_MOE_ROUTER), g.E, g.h, a.s.xm, g.h, g.B, EPI_SIGMOID_F32, a.s.scores, g.E);
  job_init(jobs[1], lptr<bf16>(a, l, KK3_MOE_LATENT_DOWN), g.lh, g.h, a.s.xm, g.h, g.B, EPI_LATENT, a.s.latent, g.lh);
  jobs[1].out2 = a.s.latent_p;
  situ_pair(a, jobs + 2, lptr<bf16>(a, l, KK3_MOE_SHARED_GATE), lptr<bf16>(a, l, KK3_MOE_SHARED_UP), g.sinter,
            a.s.shared_act);
  prepare_jobs(jobs, 4);
  return 4;
}

KK3_DEV void latent_up_job(const StepArgs& a, int l, GemvJob& j) {
  const Geo& g = a.g;
  job_init(j, lptr<bf16>(a, l, KK3_MOE_LATENT_UP), g.h, g.lh, a.s.x3, g.lh, g.B, EPI_ROUTED, a.s.prefix, g.h);
  j.aux = a.s.shared_red;
  prepare_jobs(&j, 1);
}

KK3_DEV void lm_head_job(const StepArgs& a, GemvJob& j) {
  const Geo& g = a.g;
  job_init(j, gptr<bf16>(a, KK3_LM_HEAD), g.V, g.h, a.s.xa, g.h, g.B, EPI_LOGITS, gout<float>(a, KK3_OUT_LOGITS), g.V);
  j.aux = a.s.argmax_key;
  j.aux_off = (long long)g.rank * g.V;
  prepare_jobs(&j, 1);
}

// ---- the kernel -------------------------------------------------------------------------------------

// A CTA that leaves the step because a wait ran out or an error was reported marks the step's integer outputs
// as invalid before it returns: next_token = -1 and cache_length = 0 for every row (a valid step writes a token
// in [0, vocab) and a length of 1 or context + 1). The caller learns of the failure from the outputs it reads
// after synchronising, not only from the status word at its next call. Every failing CTA writes the same
// values, and no CTA runs a later phase once the error word is set.
KK3_DEV void poison_outputs(const StepArgs& a) {
  long long* next = gout<long long>(a, KK3_OUT_NEXT_TOKEN);
  long long* len = gout<long long>(a, KK3_OUT_CACHE_LENGTH);
  for (int b = threadIdx.x; b < a.g.B; b += kThreads) {
    next[b] = -1;
    len[b] = 0;
  }
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1) kk3_step_kernel(const __grid_constant__ StepArgs a) {
  // dynamic shared memory on a 1024-byte boundary (checked below; ptxas pads the static variables before it):
  // the engines' rings of 16-byte copies assume whole 128-byte lines, and rings that straddle them ran
  // up to a third slower
  extern __shared__ __align__(1024) unsigned char smem[];
  // GEMV job descriptors live in shared memory: built once per CTA by thread 0 from the parameter block,
  // then read by every warp (indexing a per-thread array would put it in local memory)
  __shared__ GemvJob sj[kMaxJobs];
  __shared__ GemvJob sj2[2];
  __shared__ ExpertPhase sph;
  __shared__ int sjn;
  if (threadIdx.x == 0) kk3_cur_phase = 0;
  if (threadIdx.x == 0 && ((unsigned)__cvta_generic_to_shared(smem) & 1023u) != 0u) set_error(a, kErrDevice);
  __syncthreads();
  const Geo& g = a.g;
  float* fsm = reinterpret_cast<float*>(smem);
  int phase = 0;
  unsigned xi = 0;
  const unsigned seq0 = a.epoch * 1024u;
  const bool lead = threadIdx.x == 0;
  // host transport (comparison baseline): the combine and argmax phases are split at their exchange
  const bool host_comm = a.comm_mode == kCommHost && g.tp > 1;
#define KK3_RUN (phase >= a.start_phase)
#define KK3_FAIL()        \
  do {                    \
    poison_outputs(a);    \
    return;               \
  } while (0)
#define KK3_PHASE_END()                                                                      \
  do {                                                                                       \
    if (KK3_RUN && !grid_sync(a, phase)) KK3_FAIL();                                         \
    ++phase;                                                                                 \
    trace_progress(a, 0, phase);                                                             \
    if (blockIdx.x == 0 && threadIdx.x == 0 && phase <= kMaxPhases && phase > a.start_phase)             \
      a.s.phase_ts[phase] = globaltimer(); /* stamped only after phases that ran: launch ranges keep theirs */ \
    if (phase == a.stop_phase) return;                                                       \
  } while (0)
#define KK3_BUILD(stmt)   \
  do {                    \
    if (lead) { stmt; }   \
    __syncthreads();      \
  } while (0)

  if (blockIdx.x == 0 && threadIdx.x == 0) a.s.phase_ts[0] = globaltimer();
  trace_progress(a, 0, 0);
  // embedding (kimi.py:249-252)
  if (KK3_RUN) {
    prefetch_row_inputs(a, 0, 0);
    phase_embed(a, seq0 + xi, xi & 1, fsm);
  }
  int pending = PEND_EMBED;
  bool pend_signal = false;
  unsigned pend_x = xi++;
  KK3_PHASE_END();

  int nb = 0, kidx = 0, midx = 0;
  #pragma unroll 1
  for (int l = 0; l < g.L; ++l) {
    const bool mla = layer_is_mla(g, l);
    // attention prologue (kimi.py:257-262)
    if (KK3_RUN && !phase_attn_prologue(a, l, nb, pending, pend_signal, seq0 + pend_x, pend_x & 1, fsm, phase)) KK3_FAIL();
    pending = PEND_NONE;
    if (l % g.bs == 0) ++nb;
    KK3_PHASE_END();
    if (KK3_RUN) {
      KK3_BUILD(sjn = attn_proj_jobs(a, l, mla, sj));
      if (!mla) kda_state_prefetch(a, l);   // the next phase's recurrent states into L2
      if (!gemv_pass<NT>(a, sj, sjn, 0, 0, phase)) KK3_FAIL();
    }
    KK3_PHASE_END();
    if (!mla) {
      // short conv + gated delta rule (kimi.py:286-299); then prefetch the o projection into L2
      if (KK3_RUN) {
        KK3_BUILD(o_job(a, l, sj2[0]));
        #pragma unroll 1
        for (int it = blockIdx.x; it < g.B * g.hr; it += gridDim.x) kda_item(a, l, kidx, it / g.hr, it % g.hr, fsm);
        prefetch_jobs(sj2, 1);
      }
      ++kidx;
      KK3_PHASE_END();
    } else {
      if (KK3_RUN) phase_mla_rows(a, l, midx, fsm);
      KK3_PHASE_END();
      // q_b (kimi.py:265)
      if (KK3_RUN) {
        KK3_BUILD({
          job_init(sj[0], lptr<bf16>(a, l, KK3_MLA_QB), g.hr * (g.nr + g.rd), g.qr, a.s.mla_qan, g.qr, g.B,
                   EPI_STORE_BF16, a.s.mla_q, g.hr * (g.nr + g.rd));
          prepare_jobs(sj, 1);
        });
        if (!gemv_pass<NT>(a, sj, 1, 0)) KK3_FAIL();
      }
      KK3_PHASE_END();
      // absorbed query (kimi.py:271-272)
      if (KK3_RUN)
        #pragma unroll 1
        for (int it = blockIdx.x; it < g.hr * 4; it += gridDim.x) mla_absorb_item(a, l, it / 4, it % 4, fsm);
      KK3_PHASE_END();
      // split-K attention over [cache, new token] (kimi.py:274-280)
      if (KK3_RUN) {
        int total = 0;
        #pragma unroll 1
        for (int b = 0; b < g.B; ++b) total += mla_row_chunks(a, b);
        total *= g.mla_groups;
        #pragma unroll 1
        for (int it = blockIdx.x; it < total; it += gridDim.x) {
          // item -> (batch row, chunk, head group); the groups of one chunk are adjacent items, so the second
          // read of the chunk's cache rows comes from L2
          const int grp = it % g.mla_groups;
          int b = 0, rem = it / g.mla_groups;
          for (; b < g.B; ++b) {
            const int n = mla_row_chunks(a, b);
            if (rem < n) break;
            rem -= n;
          }
          const int T = mla_row_len(a, b) + 1;
          const int p0 = rem * g.mla_chunk_len;
          int p1 = p0 + g.mla_chunk_len;
          p1 = p1 < T ? p1 : T;
          const int h0 = grp * g.mla_mt * 16;
          // one instantiation per head-tile count of a group: accumulators sized exactly, three stages
          switch (g.mla_mt) {
            case 1: mla_attend_item<1, 3>(a, l, midx, b, rem, p0, p1, T, h0, smem, phase); break;
            case 2: mla_attend_item<2, 3>(a, l, midx, b, rem, p0, p1, T, h0, smem, phase); break;
            case 3: mla_attend_item<3, 3>(a, l, midx, b, rem, p0, p1, T, h0, smem, phase); break;
            default: mla_attend_item<4, 3>(a, l, midx, b, rem, p0, p1, T, h0, smem, phase); break;
          }
        }
      }
      KK3_PHASE_END();
      if (KK3_RUN) {
        KK3_BUILD(o_job(a, l, sj2[0]));
        #pragma unroll 1
        if (g.B * g.hr <= (int)gridDim.x) {
          // one item per (row, head) fits one wave
          #pragma unroll 1
          for (int it = blockIdx.x; it < g.B * g.hr; it += gridDim.x) mla_combine_row_item(a, l, it / g.hr, it % g.hr, fsm);
        } else {
          const int groups = mla_combine_groups(g.hr, g.B, gridDim.x);
          const int per = (g.B + groups - 1) / groups;   // rows per group (<= kCombRows)
          #pragma unroll 1
          for (int it = blockIdx.x; it < g.hr * groups; it += gridDim.x) {
            const int hh = it / groups, r0 = (it % groups) * per;
            const int nr = g.B - r0 < per ? g.B - r0 : per;
            if (nr <= 0) continue;
            switch (per) {   // rows per group: 1, 2, 4 or 8 (R >= per)
              case 1: mla_combine_item<1>(a, l, hh, r0, nr, smem, phase); break;
              case 2: mla_combine_item<2>(a, l, hh, r0, nr, smem, phase); break;
              case 3: case 4: mla_combine_item<4>(a, l, hh, r0, nr, smem, phase); break;
              default: mla_combine_item<8>(a, l, hh, r0, nr, smem, phase); break;
            }
          }
        }
        prefetch_jobs(sj2, 1);
      }
      ++midx;
      KK3_PHASE_END();
    }
    // o projection -> exchange
    if (KK3_RUN) {
      KK3_BUILD(o_job(a, l, sj[0]));
      prefetch_row_inputs(a, 1, l);
      if (!gemv_pass<NT>(a, sj, 1, xi & 1)) KK3_FAIL();
      if (g.tp > 1) __threadfence_system();
    }
    const unsigned x_att = xi++;
    KK3_PHASE_END();
    if (KK3_RUN && !phase_mlp_prologue(a, l, nb, seq0 + x_att, x_att & 1, fsm)) KK3_FAIL();
    KK3_PHASE_END();
    if (l < g.first_dense) {
      // dense FFN (kimi.py:304)
      if (KK3_RUN) {
        KK3_BUILD(sjn = mlp_in_jobs(a, l, sj));
        if (!gemv_pass<NT>(a, sj, sjn, 0)) KK3_FAIL();
      }
      KK3_PHASE_END();
      if (KK3_RUN) {
        KK3_BUILD({
          job_init(sj[0], lptr<bf16>(a, l, KK3_DENSE_DOWN), g.h, g.dinter, a.s.dense_act, g.dinter, g.B, EPI_EXCHANGE,
                   nullptr, g.h);
          sj[0].aux_off = a.comm.att_off;
          prepare_jobs(sj, 1);
        });
        prefetch_row_inputs(a, 0, l + 1);
        if (!gemv_pass<NT>(a, sj, 1, xi & 1)) KK3_FAIL();
        if (g.tp > 1) __threadfence_system();
      }
      pending = PEND_DENSE;
      pend_signal = true;
      pend_x = xi++;
      KK3_PHASE_END();
    } else {
      // router, latent down and the shared expert's gate/up in one pass (kimi.py:308, :317, :326)
      if (KK3_RUN) {
        KK3_BUILD(sjn = mlp_in_jobs(a, l, sj));
        // the router bias is read by every CTA at the start of the next phase: bring it into L2 now
        if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0 && g.E * 4 >= 16) {
          const float* rb = lptr<float>(a, l, KK3_MOE_ROUTER_BIAS);
          if ((reinterpret_cast<uintptr_t>(rb) & 15u) == 0) prefetch_l2(rb, (unsigned)(g.E * 4) & ~15u);
        }
        if (!gemv_pass<NT>(a, sj, sjn, 0, 0, phase)) KK3_FAIL();
      }
      KK3_PHASE_END();
      const unsigned x_moe = xi++;
      // routed experts (kimi.py:317-323); descriptor built once per CTA in shared memory
      if (KK3_RUN) {
        KK3_BUILD({
          sph.codes[0] = lptr<uint8_t>(a, l, KK3_MOE_GATE_BLOCKS);
          sph.codes[1] = lptr<uint8_t>(a, l, KK3_MOE_UP_BLOCKS);
          sph.scales[0] = lptr<uint8_t>(a, l, KK3_MOE_GATE_SCALES);
          sph.scales[1] = lptr<uint8_t>(a, l, KK3_MOE_UP_SCALES);
          sph.rows = g.inter; sph.K = g.lh; sph.tiles = g.inter / 16; sph.ksteps = g.lh / 64;
          sph.expert_codes = (long long)g.inter * g.lh / 2; sph.expert_scales = (long long)g.inter * g.lh / 32;
        });
        // every CTA routes all rows (identical tables), then the experts start (kimi.py:309-316)
        route_cta(a, l, smem, phase);
        run_experts<2>(a, sph);
      }
      KK3_PHASE_END();
      if (KK3_RUN) {
        KK3_BUILD({
          // row pairs (two 16-row tiles per unit) where the pair's scales fit the two-matrix scale layout: a
          // 16-byte window per row (K % 512 == 0) or the tile's whole block (K <= 512)
          const bool rp = down_row_pairs(g);
          sph.codes[0] = sph.codes[1] = lptr<uint8_t>(a, l, KK3_MOE_DOWN_BLOCKS);
          sph.scales[0] = sph.scales[1] = lptr<uint8_t>(a, l, KK3_MOE_DOWN_SCALES);
          if (rp) {
            sph.codes[1] += (size_t)16 * (g.inter / 2);
            sph.scales[1] += (size_t)16 * (g.inter / 32);
          }
          sph.rows = g.lh; sph.K = g.inter; sph.tiles = g.lh / (rp ? 32 : 16); sph.ksteps = g.inter / 64;
          sph.expert_codes = (long long)g.lh * g.inter / 2; sph.expert_scales = (long long)g.lh * g.inter / 32;
          job_init(sj[0], lptr<bf16>(a, l, KK3_MOE_SHARED_DOWN), g.h, g.sinter, a.s.shared_act, g.sinter, g.B,
                   EPI_EXCHANGE, nullptr, g.h);
          sj[0].aux_off = a.comm.shd_off;
          prepare_jobs(sj, 1);
        });
        // the shared expert's down projection first (kimi.py:326), then the routed experts' (:320-323); the
        // routed experts' fix-up uses counter bank 0, so this one takes bank 1
        prefetch_row_inputs(a, 2, l);
        if (!gemv_pass<NT>(a, sj, 1, x_moe & 1, 1)) KK3_FAIL();
        if (g.tp > 1) __threadfence_system();
        if (blockIdx.x == 0 && threadIdx.x == 0) sub_stamp(a, phase, 0);
        if (down_row_pairs(g)) run_experts<2, true>(a, sph);
        else run_experts<1>(a, sph);
      }
      KK3_PHASE_END();
      if (host_comm) {
        // host transport: write this rank's slots, end the phase (the host all-reduces), then read
        if (KK3_RUN && !phase_moe_combine(a, l, seq0 + x_moe, x_moe & 1, fsm, kCombineWrite)) KK3_FAIL();
        KK3_PHASE_END();
        if (KK3_RUN && !phase_moe_combine(a, l, seq0 + x_moe, x_moe & 1, fsm, kCombineRead)) KK3_FAIL();
      } else {
        if (KK3_RUN && !phase_moe_combine(a, l, seq0 + x_moe, x_moe & 1, fsm, kCombineAll)) KK3_FAIL();
      }
      KK3_PHASE_END();
      // latent up + shared + residual (kimi.py:325-329)
      if (KK3_RUN) {
        KK3_BUILD(latent_up_job(a, l, sj[0]));
        prefetch_row_inputs(a, 0, l + 1);
        if (!gemv_pass<NT>(a, sj, 1, 0)) KK3_FAIL();
      }
      KK3_PHASE_END();
    }
  }
  // head (kimi.py:330-334)
  if (pending != PEND_NONE) {
    // the last layer was dense: fold its exchange into prefix first
    if (KK3_RUN && !phase_fold_pending(a, pending, pend_signal, seq0 + pend_x, pend_x & 1)) KK3_FAIL();
    KK3_PHASE_END();
  }
  if (KK3_RUN) phase_head_prologue(a, nb, fsm);
  KK3_PHASE_END();
  if (KK3_RUN) {
    KK3_BUILD(lm_head_job(a, sj[0]));
    if (!gemv_pass<NT>(a, sj, 1, 0)) KK3_FAIL();
  }
  KK3_PHASE_END();
  const unsigned x_key = xi++;
  if (host_comm) {
    if (KK3_RUN && !phase_argmax(a, seq0 + x_key, x_key & 1, kCombineWrite)) KK3_FAIL();
    KK3_PHASE_END();
    if (KK3_RUN && !phase_argmax(a, seq0 + x_key, x_key & 1, kCombineRead)) KK3_FAIL();
  } else {
    if (KK3_RUN && !phase_argmax(a, seq0 + x_key, x_key & 1, kCombineAll)) KK3_FAIL();
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (phase + 1 <= kMaxPhases) a.s.phase_ts[phase + 1] = globaltimer();
    *a.s.phase_count = phase + 1;
  }
#undef KK3_BUILD
#undef KK3_FAIL
#undef KK3_PHASE_END
#undef KK3_RUN
}

}  // namespace kk3

