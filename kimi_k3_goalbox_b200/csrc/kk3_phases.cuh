// kk3_phases.cuh - the non-GEMV phases of the decode step: per-row residual mixing and norms, the
// one-shot tensor-parallel exchanges, KDA (gated delta rule), MLA (absorbed latent attention, split-K),
// routing.
#pragma once

#include "kk3_gemv.cuh"

namespace kk3 {

// ------------------------------------------------------------------------------------------------
// One-shot exchange over NVLink peer memory. Rank r writes its partial for batch row b into slot [r] of
// every rank's region; the writer then publishes flag [b][r] = seq on every rank (release, system scope);
// the reader acquires all tp flags of row b and sums the slots in rank order (FP32, kimi.py:343-347), so
// every rank obtains bit-identical sums. Data regions alternate by exchange parity; flags carry a
// monotonically increasing sequence number, so nothing is ever cleared.

KK3_DEV unsigned* flag_ptr(const StepArgs& a, int dst, int b, int src) {
  return reinterpret_cast<unsigned*>(a.comm.base[dst] + a.comm.flag_off) + (size_t)b * a.g.tp + src;
}

// called by a whole CTA after its writes of row b (all threads), tp > 1 only. With the host transport the
// launch ends before the slots are read and the host reduces them: nothing to signal or wait for.
KK3_DEV void xch_signal_row(const StepArgs& a, int b, unsigned seq) {
  if (a.comm_mode == kCommHost) return;
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < a.g.tp) st_release_sys(flag_ptr(a, threadIdx.x, b, a.g.rank), seq);
}

KK3_DEV bool xch_wait_row(const StepArgs& a, int b, unsigned seq) {
  if (a.comm_mode == kCommHost) return true;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < a.g.tp) {
    if (!wait_flag_sys(a, flag_ptr(a, a.g.rank, b, threadIdx.x), seq)) ok = 0;
  }
  __syncthreads();
  return ok != 0;
}

// Push transport (kCommPush). The GEMV epilogue stored this rank's partial only into its own slot of its own
// buffer; at the start of the phase that reads it every CTA copies its 1/G share of that slot (contiguous 16-byte
// pieces, read from L2) into the same slot of every peer's buffer, fences, and raises flag [rank][cta] = seq in
// each peer's chunk-push flag array. A reader waits for all G flags of every peer. Many SMs each send a few KB,
// instead of the epilogues' stores going out from whichever warps finish tiles.
KK3_DEV unsigned* push_flag_ptr(const StepArgs& a, int dst, int src, int cta) {
  return reinterpret_cast<unsigned*>(a.comm.base[dst] + a.comm.push_flag_off) + (size_t)src * gridDim.x + cta;
}
// this CTA's 1/G share of this rank's slot (sub-region `off`, slot_bytes a multiple of 16) into every peer
KK3_DEV void xch_push_stores(const StepArgs& a, int parity, long long off, long long slot_bytes) {
  const Geo& g = a.g;
  const long long n16 = slot_bytes >> 4;
  const long long c0 = n16 * blockIdx.x / gridDim.x, c1 = n16 * (blockIdx.x + 1) / gridDim.x;
  const size_t mine = (size_t)a.comm.data_off[parity] + off + (size_t)g.rank * slot_bytes;
  const uint4* src = reinterpret_cast<const uint4*>(a.comm.base[g.rank] + mine);
  for (long long i = c0 + threadIdx.x; i < c1; i += kThreads) {
    const uint4 v = __ldcg(src + i);
    #pragma unroll 1
    for (int dst = 0; dst < g.tp; ++dst)
      if (dst != g.rank) reinterpret_cast<uint4*>(a.comm.base[dst] + mine)[i] = v;
  }
}
// a whole CTA, after its stores: flag [rank][cta] = seq in the chunk flag array of every rank in [lo, hi) except
// (when skip_self) this one
KK3_DEV void xch_push_flags(const StepArgs& a, unsigned seq, bool skip_self) {
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < a.g.tp && !(skip_self && (int)threadIdx.x == a.g.rank))
    st_release_sys(push_flag_ptr(a, threadIdx.x, a.g.rank, blockIdx.x), seq);
}
// all CTAs: push this rank's slot of sub-region `off` and flag it
KK3_DEV void xch_push(const StepArgs& a, int parity, long long off, long long slot_bytes, unsigned seq) {
  xch_push_stores(a, parity, off, slot_bytes);
  xch_push_flags(a, seq, true);
}
// a whole CTA: wait until every peer's (and with self, this rank's too) every CTA flagged exchange `seq`
KK3_DEV bool xch_wait_push(const StepArgs& a, unsigned seq, bool self = false) {
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  const int n = a.g.tp * (int)gridDim.x;
  for (int i = threadIdx.x; i < n; i += kThreads) {
    const int src = i / (int)gridDim.x, cta = i - src * (int)gridDim.x;
    if ((self || src != a.g.rank) && !wait_flag_sys(a, push_flag_ptr(a, a.g.rank, src, cta), seq)) ok = 0;
  }
  __syncthreads();
  return ok != 0;
}

// local region (this rank's buffer), parity p, byte offset `off`
template <typename T>
KK3_DEV const T* xlocal(const StepArgs& a, int parity, long long off) {
  return reinterpret_cast<const T*>(a.comm.base[a.g.rank] + a.comm.data_off[parity] + off);
}

// ------------------------------------------------------------------------------------------------
// Row phases: one CTA per batch row, vectorised (16-byte loads of 8 BF16), each input read once into
// registers, all row statistics reduced in one CTA-wide pass.

constexpr int kMaxBlocks = 9;        // block vectors + prefix mixed by one attention residual (<= 8 + 1)
constexpr int kRowChunks = 2;        // 16-byte chunks per thread: rows up to 2 * 512 * 8 = 8192 elements

KK3_DEV void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
KK3_DEV uint4 pack8(const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// Row-phase staging: block vectors go to dynamic shared memory after the reduction scratch.
constexpr int kRowStageOff = 2048;   // bytes; the block_sums scratch (red) uses < 1.5 KB
KK3_DEV void cp_async16_row(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem_dst)),
               "l"(src) : "memory");
}
KK3_DEV void cp_async_commit_row() { asm volatile("cp.async.commit_group;" ::: "memory"); }
KK3_DEV void cp_async_wait_row() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// CTA-wide sums of the first `live` of N per-thread values (all threads receive the totals).
// `red`: (kWarps + 1) * N floats. Warp partials go to shared memory, warp 0 adds them, one broadcast back.
template <int N>
KK3_DEV void block_sums(float (&v)[N], float* red, int live = N) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < live) v[i] = warp_sum(v[i]);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i < live) red[warp * N + i] = v[i];
  }
  __syncthreads();
  if (warp == 0 && lane < live) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) t += red[w * N + lane];
    red[kWarps * N + lane] = t;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i < live) v[i] = red[kWarps * N + i];
}

// Block attention residual (kimi.py:199-204) then RMSNorm (common.py:13-21), for batch row b:
// hidden = bf16(sum_i softmax_i(rms(v_i) . (norm*proj)) v_i) over v = [blocks[0..nb), prefix];
// out = bf16(bf16(hidden * rsqrt(mean(hidden^2) + eps)) * ln). `pre` holds this thread's prefix chunks.
KK3_FN void mix_and_norm_regs(const StepArgs& a, int b, int nb, const uint4 (&pre)[kRowChunks], const bf16* norm,
                               const bf16* proj, const bf16* ln, float eps, bf16* out_row, float* red, int ph = -1) {
  const Geo& g = a.g;
  const int tid = threadIdx.x, nvec = g.h / 8;
  const bool stamp = ph >= 0 && b == 0 && tid == 0;
  float hidden[kRowChunks][8];
  // the final norm's weights are needed last; their load is issued first
  uint4 lnw[kRowChunks];
#pragma unroll
  for (int q = 0; q < kRowChunks; ++q) {
    const int c = tid + q * kThreads;
    lnw[q] = c < nvec ? __ldg(reinterpret_cast<const uint4*>(ln) + c) : make_uint4(0, 0, 0, 0);
  }
  if (nb > 0) {
    // every block vector this thread needs is staged into shared memory with one round of cp.async (each
    // thread reads back only its own chunks, so no CTA barrier is needed); the statistics and the mix then
    // read shared memory instead of issuing dependent L2 loads block after block
    uint4* stage = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(red) + kRowStageOff);
#pragma unroll 1
    for (int i = 0; i < nb; ++i) {
#pragma unroll
      for (int q = 0; q < kRowChunks; ++q) {
        const int c = tid + q * kThreads;
        if (c < nvec) cp_async16_row(stage + (i * kRowChunks + q) * kThreads + tid,
                                     a.s.blocks + ((size_t)i * g.B + b) * g.h + c * 8);
      }
    }
    cp_async_commit_row();
    float np[kRowChunks][8];
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) {
      const int c = tid + q * kThreads;
      float fn[8], fp[8];
      uint4 un = make_uint4(0, 0, 0, 0), up = make_uint4(0, 0, 0, 0);
      if (c < nvec) {
        un = __ldg(reinterpret_cast<const uint4*>(norm) + c);
        up = __ldg(reinterpret_cast<const uint4*>(proj) + c);
      }
      unpack8(un, fn);
      unpack8(up, fp);
#pragma unroll
      for (int e = 0; e < 8; ++e) np[q][e] = fn[e] * fp[e];
    }
    cp_async_wait_row();
    // Compact loops over the block vectors (not unrolled): this code runs once per layer with a cold
    // instruction cache, so its size, not its arithmetic, sets its time. Summation orders are those of the
    // CTA reduction used elsewhere: per thread over (chunk, element), warp shuffle tree, warps in order.
    constexpr int kSt = 2 * (kMaxBlocks + 1);
    const int warp = tid >> 5, lane = tid & 31;
    float* wred = red;                    // [kWarps][kSt] warp partials
    float* tot = red + kWarps * kSt;      // [kSt] statistics of every vector
#pragma unroll 1
    for (int i = 0; i <= nb; ++i) {
      float ss = 0.0f, dt = 0.0f;
#pragma unroll
      for (int q = 0; q < kRowChunks; ++q) {
        const int c = tid + q * kThreads;
        float f[8];
        unpack8(i == nb ? pre[q] : (c < nvec ? stage[(i * kRowChunks + q) * kThreads + tid] : make_uint4(0, 0, 0, 0)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ss += f[e] * f[e];
          dt += f[e] * np[q][e];
        }
      }
      ss = warp_sum(ss);
      dt = warp_sum(dt);
      if (lane == 0) {
        wred[warp * kSt + 2 * i] = ss;
        wred[warp * kSt + 2 * i + 1] = dt;
      }
    }
    if (stamp) sub_stamp(a, ph, 1);
    __syncthreads();
    if (tid < 2 * (nb + 1)) {
      float t = 0.0f;
#pragma unroll 1
      for (int w = 0; w < kWarps; ++w) t += wred[w * kSt + tid];
      tot[tid] = t;
    }
    __syncthreads();
    if (stamp) sub_stamp(a, ph, 2);
    // softmax over the nb + 1 logits rms(v_i) . (norm * proj), then the weighted sum
    float mx = -INFINITY;
#pragma unroll 1
    for (int i = 0; i <= nb; ++i) mx = fmaxf(mx, tot[2 * i + 1] * rsqrtf(tot[2 * i] / (float)g.h + 1e-5f));
    float den = 0.0f;
#pragma unroll 1
    for (int i = 0; i <= nb; ++i) den += expf(tot[2 * i + 1] * rsqrtf(tot[2 * i] / (float)g.h + 1e-5f) - mx);
    float accv[kRowChunks][8];
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e) accv[q][e] = 0.0f;
#pragma unroll 1
    for (int i = 0; i <= nb; ++i) {
      const float pi = expf(tot[2 * i + 1] * rsqrtf(tot[2 * i] / (float)g.h + 1e-5f) - mx) / den;
#pragma unroll
      for (int q = 0; q < kRowChunks; ++q) {
        const int c = tid + q * kThreads;
        float f[8];
        unpack8(i == nb ? pre[q] : (c < nvec ? stage[(i * kRowChunks + q) * kThreads + tid] : make_uint4(0, 0, 0, 0)), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) accv[q][e] += pi * f[e];
      }
    }
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e) hidden[q][e] = round_bf(accv[q][e]);
  } else {
#pragma unroll
    for (int q = 0; q < kRowChunks; ++q) unpack8(pre[q], hidden[q]);
  }
  float ss[1] = {0.0f};
#pragma unroll
  for (int q = 0; q < kRowChunks; ++q)
#pragma unroll
    for (int e = 0; e < 8; ++e) ss[0] += hidden[q][e] * hidden[q][e];
  if (stamp) sub_stamp(a, ph, 3);
  block_sums<1>(ss, red + (kWarps + 1) * 2 * (kMaxBlocks + 1));
  if (stamp) sub_stamp(a, ph, 4);
  const float rs = rsqrtf(ss[0] / (float)g.h + eps);
#pragma unroll
  for (int q = 0; q < kRowChunks; ++q) {
    const int c = tid + q * kThreads;
    if (c < nvec) {
      float w[8], o[8];
      unpack8(lnw[q], w);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = round_bf(round_bf(hidden[q][e] * rs) * w[e]);
      *reinterpret_cast<uint4*>(out_row + c * 8) = pack8(o);
    }
  }
  if (stamp) sub_stamp(a, ph, 5);
}

// RMSNorm of one BF16 row of width n <= 8192 (common.py:13-21), vectorised
KK3_FN void rms_row(const bf16* in, const bf16* w, int n, float eps, bf16* out, float* red) {
  const int nvec = n / 8;
  float x[kRowChunks][8];
  float ss[1] = {0.0f};
#pragma unroll
  for (int q = 0; q < kRowChunks; ++q) {
    const int c = threadIdx.x + q * kThreads;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (c < nvec) v = ld_act16(in + c * 8);
    unpack8(v, x[q]);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss[0] += x[q][e] * x[q][e];
  }
  block_sums<1>(ss, red);
  const float rs = rsqrtf(ss[0] / (float)n + eps);
#pragma unroll
  for (int q = 0; q < kRowChunks; ++q) {
    const int c = threadIdx.x + q * kThreads;
    if (c < nvec) {
      float wf[8], o[8];
      unpack8(ld_act16(w + c * 8), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = round_bf(round_bf(x[q][e] * rs) * wf[e]);
      *reinterpret_cast<uint4*>(out + c * 8) = pack8(o);
    }
  }
  __syncthreads();
}

// Sum of the tp bf16 slots of row b, 16-byte chunk c (channels 8c .. 8c + 7, layout xch_index), in FP32 and
// rank order, rounded to BF16 (kimi.py:343-347). With the host transport the host has
// already all-reduced the partials into this rank's own slot (FP32 sum, cast to bf16), so that slot is read.
KK3_DEV void xch_sum8(const StepArgs& a, int parity, long long off, int b, int width, int c, float (&out)[8]) {
  const bf16* base = xlocal<bf16>(a, parity, off);
#pragma unroll
  for (int e = 0; e < 8; ++e) out[e] = 0.0f;
  const int lo = a.comm_mode == kCommHost ? a.g.rank : 0, hi = a.comm_mode == kCommHost ? a.g.rank + 1 : a.g.tp;
  for (int src = lo; src < hi; ++src) {
    float f[8];
    unpack8(ld_act16(base + xch_index(a.g, src, b, c * 8, width)), f);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] += f[e];
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) out[e] = round_bf(out[e]);
}

// ------------------------------------------------------------------------------------------------
// KDA: one CTA per (batch row, head). Short convolution (kimi.py:286-289), f_a/f_b gate (:290),
// beta (:291), gated delta rule on the V-first FP32 state (:207-215), gated per-head RMSNorm (:296-298).

KK3_FN void kda_item(const StepArgs& a, int layer, int kidx, int b, int hh, float* sm) {
  const Geo& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int D = g.qdim, dh = 128;
  float* sq = sm;            // [128] q after conv
  float* sk = sm + 128;      // [128] k after conv
  float* sv = sm + 256;      // [128] v after conv
  float* decay = sm + 384;   // [128]
  float* qn = sm + 512;      // [128]
  float* kn = sm + 640;      // [128]
  float* outv = sm + 768;    // [128]
  float* fa = sm + 896;      // [128]
  float* misc = sm + 1024;   // [32]
  const bool stamp = blockIdx.x == 0 && tid == 0;   // profiling stamps of CTA 0's first item (sub 0-5)
  if (stamp) sub_stamp(a, kk3_cur_phase, 0);
  const bool keep = !reinterpret_cast<const bool*>(a.ptr[KK3_RESET])[b];
  const bf16* conv_in = lptr<bf16>(a, layer, KK3_KDA_CONV_STATE);
  const float* cw = lptr<float>(a, layer, KK3_KDA_CONV_WEIGHT);
  bf16* conv_out = gout<bf16>(a, KK3_OUT_CONV_STATE) + (size_t)kidx * g.B * 3 * D * 4;
  const float* st_in = lptr<float>(a, layer, KK3_KDA_RECURRENT_STATE) + (((size_t)b * g.hr + hh) * dh) * dh;
  float* st_out = gout<float>(a, KK3_OUT_RECURRENT_STATE) + ((((size_t)kidx * g.B + b) * g.hr + hh) * dh) * dh;

  // An item is a chain of short dependent steps, so every global load that needs no result of this item is
  // issued first and their latencies overlap: this warp's eight state rows, this thread's quarter of an f_b
  // row, the conv inputs and weights, the decay parameters and the output gate.
  float4 rows[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    rows[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (keep) rows[i] = *reinterpret_cast<const float4*>(st_in + (size_t)(warp * 8 + i) * dh + lane * 4);
  }
  // f_b (kimi.py:290): output channel gd = tid / 4; part gp sums the 8-wide input chunks gp, gp + 4, gp + 8 and
  // gp + 12, so the four parts of a channel read 64 contiguous bytes per load and distinct shared-memory banks
  const int gd = tid >> 2, gp = tid & 3;
  const uint4* fbp = reinterpret_cast<const uint4*>(lptr<bf16>(a, layer, KK3_KDA_FB) + (size_t)(hh * dh + gd) * dh);
  uint4 fbw[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) fbw[q] = fbp[q * 4 + gp];
  const float A = gp == 0 ? expf(lptr<float>(a, layer, KK3_KDA_A_LOG)[hh]) : 0.0f;
  const float dtb = gp == 0 ? lptr<float>(a, layer, KK3_KDA_DT_BIAS)[hh * dh + gd] : 0.0f;
  // conv (kimi.py:286-289): thread (i, dd) of the first 384 holds channel dd of q, k or v
  const int ci = tid >> 7, cd = tid & 127;
  const size_t coff = (((size_t)b * 3 + ci) * D + hh * dh + cd) * 4;
  float raw = 0.0f, w1 = 0.0f, w2 = 0.0f, w3 = 0.0f;
  float4 cwv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (tid < 384) {
    raw = bf2f(a.s.qkv[((size_t)b * 3 + ci) * D + hh * dh + cd]);
    if (keep) {
      w1 = bf2f(conv_in[coff + 1]);
      w2 = bf2f(conv_in[coff + 2]);
      w3 = bf2f(conv_in[coff + 3]);
    }
    cwv = *reinterpret_cast<const float4*>(cw + ((size_t)ci * D + hh * dh + cd) * 4);
  }
  float ogt[4] = {0.0f, 0.0f, 0.0f, 0.0f};   // warp 0: output gate of value channels 4 lane .. 4 lane + 3
  if (warp == 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) ogt[q] = bf2f(a.s.og[(size_t)b * D + hh * dh + lane * 4 + q]);
  }
  if (tid < 128) fa[tid] = bf2f(a.s.fa[(size_t)b * dh + tid]);
  __syncthreads();
  if (stamp) sub_stamp(a, kk3_cur_phase, 1);
  {
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const bf16* wv = reinterpret_cast<const bf16*>(&fbw[q]);
      const float4 f0 = *reinterpret_cast<const float4*>(fa + (q * 4 + gp) * 8);
      const float4 f1 = *reinterpret_cast<const float4*>(fa + (q * 4 + gp) * 8 + 4);
      acc += bf2f(wv[0]) * f0.x + bf2f(wv[1]) * f0.y + bf2f(wv[2]) * f0.z + bf2f(wv[3]) * f0.w +
             bf2f(wv[4]) * f1.x + bf2f(wv[5]) * f1.y + bf2f(wv[6]) * f1.z + bf2f(wv[7]) * f1.w;
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    if (gp == 0) decay[gd] = expf(-5.0f * sigmoidf_(A * (round_bf(acc) + dtb)));
  }
  if (tid < 384) {
    bf16* co = conv_out + coff;
    co[0] = f2bf(w1);
    co[1] = f2bf(w2);
    co[2] = f2bf(w3);
    co[3] = f2bf(raw);
    const float s = w1 * cwv.x + w2 * cwv.y + w3 * cwv.z + raw * cwv.w;
    const float act = round_bf(s * sigmoidf_(s));
    (ci == 0 ? sq : (ci == 1 ? sk : sv))[cd] = act;
  }
  __syncthreads();
  if (stamp) sub_stamp(a, kk3_cur_phase, 2);
  if (warp < 2) {
    const float* src = warp == 0 ? sq : sk;
    float v[4], ss = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[q] = src[lane * 4 + q];
      ss += v[q] * v[q];
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss + 1e-6f);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (warp == 0) qn[lane * 4 + q] = v[q] * rs / 11.313708498984761f;
      else kn[lane * 4 + q] = v[q] * rs;
    }
  } else if (warp == 2 && lane == 0) {
    misc[0] = sigmoidf_(bf2f(a.s.beta[(size_t)b * g.hr + hh]));
  }
  __syncthreads();
  if (stamp) sub_stamp(a, kk3_cur_phase, 3);
  const float sb = misc[0];
  const float4 dk = *reinterpret_cast<const float4*>(decay + lane * 4);
  const float4 kk = *reinterpret_cast<const float4*>(kn + lane * 4);
  const float4 qq = *reinterpret_cast<const float4*>(qn + lane * 4);
  // The warp's eight value rows are independent: their two reductions each run as one interleaved butterfly,
  // in warp_sum's xor order, so the sums are those of a row at a time.
  float pred[8], o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4& s = rows[i];
    s.x *= dk.x; s.y *= dk.y; s.z *= dk.z; s.w *= dk.w;
    pred[i] = s.x * kk.x + s.y * kk.y + s.z * kk.z + s.w * kk.w;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) pred[i] += __shfl_xor_sync(0xffffffffu, pred[i], off);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4& s = rows[i];
    const float err = (sv[warp * 8 + i] - pred[i]) * sb;
    s.x += err * kk.x; s.y += err * kk.y; s.z += err * kk.z; s.w += err * kk.w;
    o[i] = s.x * qq.x + s.y * qq.y + s.z * qq.z + s.w * qq.w;
    *reinterpret_cast<float4*>(st_out + (size_t)(warp * 8 + i) * dh + lane * 4) = s;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] += __shfl_xor_sync(0xffffffffu, o[i], off);
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) outv[warp * 8 + i] = o[i];
  }
  __syncthreads();
  if (stamp) sub_stamp(a, kk3_cur_phase, 4);
  if (warp == 0) {
    float o[4], ss = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      o[q] = round_bf(outv[lane * 4 + q]);
      ss += o[q] * o[q];
    }
    ss = warp_sum(ss);
    const float rs = rsqrtf(ss / 128.0f + 1e-5f);
    const float* onorm = lptr<float>(a, layer, KK3_KDA_ONORM);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int v = lane * 4 + q;
      a.s.attn_in[(size_t)b * D + hh * dh + v] = f2bf(o[q] * rs * onorm[v] * sigmoidf_(ogt[q]));
    }
  }
  __syncthreads();
  if (stamp) sub_stamp(a, kk3_cur_phase, 5);
}

// Issued by thread 0 of every CTA at the start of the KDA layer's projection phase: an L2 prefetch of the FP32
// recurrent state (64 KB per (row, head)) of each item this CTA will run in the next phase (items it =
// blockIdx + k * grid, state index it = b * hr + head), so the items' first loads hit L2 instead of HBM. Rows
// that are reset read no state.
// Only when the phase's items fit one wave: with several waves the prefetch measured no gain in the KDA phase and
// slowed the projection phase it runs in (dev-l4: +18 us per step).
KK3_FN void kda_state_prefetch(const StepArgs& a, int layer) {
  const Geo& g = a.g;
  if (threadIdx.x != 0 || g.B * g.hr > (int)gridDim.x) return;
  const float* st = lptr<float>(a, layer, KK3_KDA_RECURRENT_STATE);
  const bool* reset = reinterpret_cast<const bool*>(a.ptr[KK3_RESET]);
  #pragma unroll 1
  for (int it = blockIdx.x; it < g.B * g.hr; it += gridDim.x)
    if (!reset[it / g.hr]) prefetch_l2(st + (size_t)it * 128 * 128, 128u * 128u * 4u);
}

// ------------------------------------------------------------------------------------------------
// MLA (kimi.py:263-283), absorbed latent form.

// absorbed[b, h, c] = bf16(sum_d q[b, h, d] * kb[h*256 + d, c]), d < nr   (kimi.py:271-272)
KK3_FN void mla_absorb_item(const StepArgs& a, int layer, int hh, int cq, float* sm) {
  const Geo& g = a.g;
  const int tid = threadIdx.x;
  const int c = cq * 128 + (tid & 127), dq = tid >> 7;   // 4 quarters of the 128 nope dims
  const bf16* kb = lptr<bf16>(a, layer, KK3_MLA_KB);
  float* qs = sm;                  // [B][128]
  float* part = sm + g.B * 128;    // [4][16][128]
  for (int i = tid; i < g.B * 128; i += kThreads) {
    const int b = i >> 7, d = i & 127;
    qs[i] = bf2f(a.s.mla_q[((size_t)b * g.hr + hh) * (g.nr + g.rd) + d]);
  }
  __syncthreads();
  // this thread's 32 weights (one column c, nope dims 32dq..32dq+31), all loads in flight at once
  float w[32];
  {
    const bf16* col = kb + ((size_t)hh * (g.nr + g.vd) + dq * 32) * g.kr + c;
#pragma unroll
    for (int d = 0; d < 32; ++d) w[d] = bf2f(col[(size_t)d * g.kr]);
  }
  for (int b0 = 0; b0 < g.B; b0 += 16) {
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
#pragma unroll
    for (int d = 0; d < 32; ++d) {
#pragma unroll
      for (int i = 0; i < 16; ++i)
        if (b0 + i < g.B) acc[i] += qs[(b0 + i) * 128 + dq * 32 + d] * w[d];
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) part[(dq * 16 + i) * 128 + (tid & 127)] = acc[i];
    __syncthreads();
    if (dq == 0) {
      for (int i = 0; i < 16 && b0 + i < g.B; ++i) {
        const float s = part[(0 * 16 + i) * 128 + (tid & 127)] + part[(1 * 16 + i) * 128 + (tid & 127)] +
                        part[(2 * 16 + i) * 128 + (tid & 127)] + part[(3 * 16 + i) * 128 + (tid & 127)];
        a.s.absorbed[(((size_t)(b0 + i)) * g.hr + hh) * g.kr + c] = f2bf(s);
      }
    }
    __syncthreads();
  }
}

// shared-memory layout of one attention item
constexpr int kRowDims = 576;   // 512 latent + 64 rope dims of a cached position (kv_lora_rank 512, rope 64)
constexpr int kRowK = 584;   // padded row (elements) of a cached position: 512 latent + 64 rope + 8 pad
constexpr int kRowP = 40;    // padded row of the BF16 probability tile (32 positions + 8)
constexpr int kRowS = 33;    // padded row of the FP32 score tile

// Pipeline depth (position sub-tiles in flight) and k-split of the score product for a head-tile count:
// three stages while they fit next to the query tile; the 576-wide score dot products of each (head tile,
// 8 positions) split KQ ways so that the MT x 4 x KQ score items use the 16 warps (MT = 1: 16 items of 9
// k-steps, 2: 16 of 18, 3: 12 of 36, 4: 16 of 36). Splitting MT = 3 four ways (48 items of 9, three per warp)
// measured slower (score sub-phase 2.7 against 1.7 us per 32 positions).
__host__ __device__ inline int mla_stages(int HR) { return HR <= 64 ? 3 : 2; }
__host__ __device__ constexpr int mla_kq(int MT) { return MT == 1 ? 4 : (MT == 2 ? 2 : 1); }
__host__ __device__ inline size_t mla_smem_bytes(int HR) {
  return (size_t)(HR + mla_stages(HR) * kMlaPos) * kRowK * 2 + (size_t)mla_kq(HR / 16) * HR * kRowS * 4 +
         (size_t)HR * kRowP * 2 + 3 * HR * 4 + 64;
}

KK3_DEV unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }

KK3_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
KK3_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
KK3_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
KK3_DEV void cp_async_wait_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

KK3_DEV void ldsm_x4(unsigned (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(smem_u32(p)));
}
KK3_DEV void ldsm_x2(unsigned (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
KK3_DEV void ldsm_x2_t(unsigned (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}

// stage positions [t0, t0+32) of row b (cache rows, the new token at t == ctx, zero beyond T)
// Source rows of one batch row's attended sequence: cache positions first (kept rows only), then the new
// token's latent and rope rows. Each thread stages the same (position, 16-byte piece) pattern for every
// sub-tile, so its piece offsets are computed once per item.
struct MlaSrc {
  const bf16* kv;    // kv_cache row 0 of this batch row
  const bf16* pe;    // pe_cache row 0
  const bf16* kvw;   // new token's latent row (kv_write)
  const bf16* pew;   // new token's rope row (pe_write)
  int ncache;        // cached positions attended (ctx for a kept row, 0 after a reset)
  int kr, rd;
  unsigned long long pol;   // L2 evict_first: the cache is read once per step
};

constexpr int kMlaPieces = kMlaPos * 72;                       // 16-byte pieces of one 32-position sub-tile
constexpr int kMlaPiecesPerThread = (kMlaPieces + kThreads - 1) / kThreads;

KK3_DEV void mla_stage(const MlaSrc& src, int t0, int T, bf16* dst) {
#pragma unroll
  for (int j = 0; j < kMlaPiecesPerThread; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i >= kMlaPieces) break;
    const int tl = i / 72, q = i - (i / 72) * 72, t = t0 + tl;
    bf16* d = dst + tl * kRowK + q * 8;
    if (t < src.ncache) {
      cp_async16_stream(d, q < 64 ? src.kv + (size_t)t * src.kr + q * 8 : src.pe + (size_t)t * src.rd + (q - 64) * 8,
                        src.pol);
    } else if (t < T) {
      *reinterpret_cast<uint4*>(d) = ld_act16(q < 64 ? src.kvw + q * 8 : src.pew + (q - 64) * 8);
    } else {
      *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
    }
  }
  cp_async_commit();
}

// One split-K item: batch row b, positions [p0, p1) of its attended sequence (T = ctx+1 or 1).
// Writes (m, l, O[kr]) per head for the combine phase (flash-decoding with online softmax). Position
// sub-tiles of 32 stream through an NS-deep cp.async ring; the score product S = Q K^T is split over
// (head tile, 8 positions, k-quarter) so every warp works, and the k-partials are summed in a fixed order.
template <int MT, int NS>
KK3_FN void mla_attend_item(const StepArgs& a, int layer, int midx, int b, int chunk, int p0, int p1, int T, int h0,
                            unsigned char* smem, int ph = -1) {
  const Geo& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, r = lane >> 2, c = lane & 3;
  constexpr int HR = MT * 16;
  const bool stamp = ph >= 0 && b == 0 && chunk == 0 && h0 == 0 && tid == 0;   // sub-phase stamps of one item
  if (stamp) sub_stamp(a, ph, 0);
  constexpr int KQ = mla_kq(MT), KPER = kRowDims / 16 / KQ;   // 36 k-steps of 16, split KQ ways
  bf16* Qs = reinterpret_cast<bf16*>(smem);                         // [HR][kRowK]
  bf16* Ks = Qs + HR * kRowK;                                       // [NS][32][kRowK]
  float* Sp = reinterpret_cast<float*>(Ks + NS * kMlaPos * kRowK);   // [KQ][HR][kRowS] k-partial scores
  bf16* Ps = reinterpret_cast<bf16*>(Sp + KQ * HR * kRowS);         // [HR][kRowP]
  float* mrun = reinterpret_cast<float*>(Ps + HR * kRowP);          // [HR]
  float* lrun = mrun + HR;                                          // [HR]
  float* alpha = lrun + HR;                                         // [HR]
  const float scale = rsqrtf((float)(g.nr + g.rd));
  const int Tend = p1 < T ? p1 : T;
  const int nsub = (p1 - p0 + kMlaPos - 1) / kMlaPos;
  MlaSrc src;
  src.kv = lptr<bf16>(a, layer, KK3_MLA_KV_CACHE) + (size_t)b * g.ctx * g.kr;
  src.pe = lptr<bf16>(a, layer, KK3_MLA_PE_CACHE) + (size_t)b * g.ctx * g.rd;
  src.kvw = gout<bf16>(a, KK3_OUT_KV_WRITE) + ((size_t)midx * g.B + b) * g.kr;
  src.pew = gout<bf16>(a, KK3_OUT_PE_WRITE) + ((size_t)midx * g.B + b) * g.rd;
  src.ncache = mla_row_len(a, b);
  src.pol = l2_evict_first_policy();
  src.kr = g.kr;
  src.rd = g.rd;
  // Q rows of heads h0 .. h0 + HR - 1: absorbed (512) | q rope (64), copied asynchronously in the group of the
  // first sub-tile; zero for padded heads
  for (int i = tid; i < HR * 72; i += kThreads) {
    const int hh = i / 72, q = i % 72, h = h0 + hh;
    bf16* d = Qs + hh * kRowK + q * 8;
    if (h < g.hr) {
      cp_async16(d, q < 64 ? a.s.absorbed + (((size_t)b * g.hr + h) * g.kr) + q * 8
                           : a.s.mla_q + ((size_t)b * g.hr + h) * (g.nr + g.rd) + g.nr + (q - 64) * 8);
    } else {
      *reinterpret_cast<uint4*>(d) = make_uint4(0, 0, 0, 0);
    }
  }
  // the first NS - 1 sub-tiles go out right behind it
  for (int s = 0; s < NS - 1; ++s) {
    if (s < nsub) mla_stage(src, p0 + s * kMlaPos, Tend, Ks + s * kMlaPos * kRowK);
    else cp_async_commit();
  }
  for (int i = tid; i < HR; i += kThreads) {
    mrun[i] = -INFINITY;
    lrun[i] = 0.0f;
  }
  if (stamp) sub_stamp(a, ph, 1);
  // O accumulators: warp w owns latent dims [32w, 32w+32) for every head tile
  float O[MT][4][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) O[mt][nt][i] = 0.0f;

  for (int s = 0; s < nsub; ++s) {
    const int t0 = p0 + s * kMlaPos;
    bf16* Kc = Ks + (s % NS) * kMlaPos * kRowK;
    if (s + NS - 1 < nsub)
      mla_stage(src, t0 + (NS - 1) * kMlaPos, Tend, Ks + ((s + NS - 1) % NS) * kMlaPos * kRowK);
    else
      cp_async_commit();
    if (NS == 3) asm volatile("cp.async.wait_group 2;" ::: "memory");
    else asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    if (stamp && s < 2) sub_stamp(a, ph, 2 + 4 * s);
    // k-partial scores: items (k-quarter, head tile, 8-position n-tile)
#pragma unroll 1
    for (int it = warp; it < MT * 4 * KQ; it += kWarps) {
      const int kq = it % KQ, mt = (it / KQ) >> 2, nt = (it / KQ) & 3;
      const bf16* qrow = Qs + (mt * 16 + (lane & 15)) * kRowK + kq * KPER * 16 + (lane >> 4) * 8;
      const bf16* krow = Kc + (nt * 8 + (lane & 7)) * kRowK + kq * KPER * 16 + ((lane >> 3) & 1) * 8;
      float sacc[4];
      if constexpr (MT <= 2) {
        // 9 or 18 k-steps, fully unrolled over four accumulators: the shared-memory loads of later k-steps are
        // issued while earlier MMAs run (score sub-phase 1.0 -> 0.6 us per 32 positions at MT = 1)
        float acc4[4][4];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 4; ++i) acc4[c][i] = 0.0f;
#pragma unroll
        for (int k = 0; k < KPER; ++k) {
          unsigned af[4], bfr[2];
          ldsm_x4(af, qrow + k * 16);
          ldsm_x2(bfr, krow + k * 16);
          mma_bf16(acc4[k & 3], af[0], af[1], af[2], af[3], bfr[0], bfr[1]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) sacc[i] = (acc4[0][i] + acc4[1][i]) + (acc4[2][i] + acc4[3][i]);
      } else {
        // 36 k-steps with the O accumulators of MT >= 3 head tiles live: two accumulators (even / odd k-steps),
        // not unrolled (unrolled, the registers spill)
        float s0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
        for (int k = 0; k < KPER; k += 2) {
          unsigned af[4], bfr[2];
          ldsm_x4(af, qrow + k * 16);
          ldsm_x2(bfr, krow + k * 16);
          mma_bf16(s0, af[0], af[1], af[2], af[3], bfr[0], bfr[1]);
          ldsm_x4(af, qrow + (k + 1) * 16);
          ldsm_x2(bfr, krow + (k + 1) * 16);
          mma_bf16(s1, af[0], af[1], af[2], af[3], bfr[0], bfr[1]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) sacc[i] = s0[i] + s1[i];
      }
      float* sp = Sp + (size_t)kq * HR * kRowS;
      sp[(mt * 16 + r) * kRowS + nt * 8 + 2 * c] = sacc[0];
      sp[(mt * 16 + r) * kRowS + nt * 8 + 2 * c + 1] = sacc[1];
      sp[(mt * 16 + r + 8) * kRowS + nt * 8 + 2 * c] = sacc[2];
      sp[(mt * 16 + r + 8) * kRowS + nt * 8 + 2 * c + 1] = sacc[3];
    }
    __syncthreads();
    if (stamp && s < 2) sub_stamp(a, ph, 3 + 4 * s);
    // online softmax, one warp per head row, one lane per position (k-partials summed in order)
    for (int hh = warp; hh < HR; hh += kWarps) {
      const bool valid = (t0 + lane) < p1 && (t0 + lane) < T && h0 + hh < g.hr;
      float sum = 0.0f;
      for (int q = 0; q < KQ; ++q) sum += Sp[((size_t)q * HR + hh) * kRowS + lane];
      const float sv = valid ? sum * scale : -INFINITY;
      const float mt_ = warp_max(sv);
      const float mold = mrun[hh];
      const float mnew = fmaxf(mold, mt_);
      const float p = valid ? expf(sv - mnew) : 0.0f;
      const float ps = warp_sum(p);
      Ps[hh * kRowP + lane] = f2bf(p);
      if (lane == 0) {
        const float al = (mold == -INFINITY) ? 0.0f : expf(mold - mnew);
        alpha[hh] = (mnew == -INFINITY) ? 1.0f : al;
        lrun[hh] = lrun[hh] * alpha[hh] + ps;
        mrun[hh] = mnew;
      }
    }
    __syncthreads();
    if (stamp && s < 2) sub_stamp(a, ph, 4 + 4 * s);
    // O = O * alpha + P V over this sub-tile: warp w owns dims [32w, 32w+32)
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const float a0 = alpha[mt * 16 + r], a1 = alpha[mt * 16 + r + 8];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        O[mt][nt][0] *= a0; O[mt][nt][1] *= a0; O[mt][nt][2] *= a1; O[mt][nt][3] *= a1;
      }
    }
#pragma unroll
    for (int k0 = 0; k0 < kMlaPos; k0 += 16) {
      unsigned bfr[4][2];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) ldsm_x2_t(bfr[nt], Kc + (k0 + (lane & 15)) * kRowK + warp * 32 + nt * 8);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        unsigned af[4];
        ldsm_x4(af, Ps + (mt * 16 + (lane & 15)) * kRowP + k0 + (lane >> 4) * 8);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) mma_bf16(O[mt][nt], af[0], af[1], af[2], af[3], bfr[nt][0], bfr[nt][1]);
      }
    }
    __syncthreads();
    if (stamp && s < 2) sub_stamp(a, ph, 5 + 4 * s);
  }
  cp_async_wait_all();
  if (stamp) sub_stamp(a, ph, 10);
  if (stamp) sub_stamp(a, ph, 11, (unsigned long long)nsub);
  // write the partial: [b][chunk][h] x (m, l, O[512])
  const int stride = g.kr + 2;
  float* base = a.s.mla_part + (((size_t)b * g.mla_chunks + chunk) * g.hr + h0) * stride;
  for (int hh = tid; hh < HR && h0 + hh < g.hr; hh += kThreads) {
    base[(size_t)hh * stride] = mrun[hh];
    base[(size_t)hh * stride + 1] = lrun[hh];
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int hh = mt * 16 + r + 8 * (i >> 1);
        const int col = warp * 32 + nt * 8 + 2 * c + (i & 1);
        if (h0 + hh < g.hr) base[(size_t)hh * stride + 2 + col] = O[mt][nt][i];
      }
    }
  }
  __syncthreads();
}

// Combine of one (batch row, head): used when rows x heads items fit one wave of the grid (few heads per rank),
// where it is faster than the per-head items below. Combines the split-K partials, applies kb's value half
// and the sigmoid output gate (kimi.py:280-282): out[d] = bf16(bf16(sum_c lat[c] * kb[h*256+128+d, c]) * bf16(sigmoid(og))).
KK3_FN void mla_combine_row_item(const StepArgs& a, int layer, int b, int hh, float* sm) {
  const Geo& g = a.g;
  const int tid = threadIdx.x;
  const bool keep = !reinterpret_cast<const bool*>(a.ptr[KK3_RESET])[b];
  const int nck = mla_row_chunks(a, b);
  const int stride = g.kr + 2;
  const float* base = a.s.mla_part + (((size_t)b * g.mla_chunks) * g.hr + hh) * stride;
  const size_t cstride = (size_t)g.hr * stride;
  float* lat = sm;                // [512]
  float* wgt = sm + 512;          // [chunks <= 64]
  float* misc = sm + 512 + 64;    // [2]
  float* lsum = sm + 512 + 128;   // [chunks <= 64]: l of each chunk
  if (tid < 32) {
    // warp 0: every lane loads the (m, l) of chunks lane and lane + 32 at once (a loop of dependent loads by one
    // thread took most of the item at 65 chunks); L is summed in chunk order by lane 0
    float m0 = -INFINITY, m1 = -INFINITY;
    if (tid < nck) {
      m0 = ld_cg_f32(base + tid * cstride);
      lsum[tid] = ld_cg_f32(base + tid * cstride + 1);
    }
    if (tid + 32 < nck) {
      m1 = ld_cg_f32(base + (tid + 32) * cstride);
      lsum[tid + 32] = ld_cg_f32(base + (tid + 32) * cstride + 1);
    }
    const float M = warp_max(fmaxf(m0, m1));
    if (tid < nck) wgt[tid] = (m0 == -INFINITY) ? 0.0f : expf(m0 - M);
    if (tid + 32 < nck) wgt[tid + 32] = (m1 == -INFINITY) ? 0.0f : expf(m1 - M);
    __syncwarp();
    if (tid == 0) {
      float Lsum = 0.0f;
      for (int i = 0; i < nck; ++i) Lsum += wgt[i] * lsum[i];
      misc[0] = 1.0f / Lsum;
    }
  }
  __syncthreads();
  for (int cc = tid; cc < g.kr; cc += kThreads) {
    // 16 chunk loads in flight, summed in chunk order
    float acc = 0.0f;
    for (int i0 = 0; i0 < nck; i0 += 16) {
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = i0 + k < nck ? ld_cg_f32(base + (size_t)(i0 + k) * cstride + 2 + cc) : 0.0f;
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if (i0 + k < nck) acc += wgt[i0 + k] * v[k];
    }
    lat[cc] = round_bf(acc * misc[0]);
  }
  __syncthreads();
  // the attended latent (kimi.py:280) replaces the absorbed query in scratch, for diagnostics
  for (int cc = tid; cc < g.kr; cc += kThreads)
    a.s.absorbed[(((size_t)b) * g.hr + hh) * g.kr + cc] = f2bf(lat[cc]);
  // value projection: 4 threads per output dim, 128 latent dims each
  const bf16* kb = lptr<bf16>(a, layer, KK3_MLA_KB);
  const int dv = tid >> 2, part = tid & 3;
  float acc = 0.0f;
  if (dv < g.vd) {
    const bf16* row = kb + ((size_t)hh * (g.nr + g.vd) + g.nr + dv) * g.kr + part * 128;
    for (int e = 0; e < 128; e += 8) {
      const uint4 w = *reinterpret_cast<const uint4*>(row + e);
      const bf16* wv = reinterpret_cast<const bf16*>(&w);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc += bf2f(wv[q]) * lat[part * 128 + e + q];
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  if (dv < g.vd && part == 0) {
    const float o = round_bf(acc);
    const float gt = round_bf(sigmoidf_(bf2f(a.s.og[(size_t)b * g.hr * g.vd + hh * g.vd + dv])));
    a.s.attn_in[(size_t)b * g.hr * g.vd + hh * g.vd + dv] = f2bf(o * gt);
  }
  __syncthreads();
}

// Combine the split-K partials and apply kb's value half with the sigmoid output gate (kimi.py:280-282):
// out[d] = bf16(bf16(sum_c lat[c] * kb[h*256+128+d, c]) * bf16(sigmoid(og))). One item is a head and a group of
// batch rows (groups chosen so that heads x groups fills the grid), so every attended latent is formed once:
//  1. per row (one warp each, all chunk loads at once): weights exp(m_i - M) and 1/L, summed in chunk order;
//  2. lat[b][c] = bf16(sum_i w_i O_i[c] / L) into shared memory (bf16 is exact: the reference rounds it),
//     thread = latent dim, 32 loads in flight at a time whatever the group's row count;
//  3. out[b][d] = sum_c lat[b][c] kb[d][c] in two passes of 64 output dims: 8 threads per dim, 64 latent dims
//     each (weights in registers), partials reduced across the 8 threads.
constexpr int kCombRow = 72;   // bf16 per (row, 64-dim part) of the latent tile: 64 + 8 pad (bank offsets)
constexpr int kCombRows = 8;   // rows per item at most
__host__ __device__ inline size_t mla_combine_smem_bytes(int B) {
  const int R = B < kCombRows ? B : kCombRows;
  return (size_t)R * 8 * kCombRow * 2 + (size_t)R * 128 * 4 + (size_t)R * 4 + 64;
}
// batch-row groups per head: enough items for the grid, groups of at most kCombRows rows
__host__ __device__ inline int mla_combine_groups(int hr, int B, int grid) {
  int n = grid / (hr > 0 ? hr : 1);
  const int need = (B + kCombRows - 1) / kCombRows;
  n = n < need ? need : (n > B ? B : n);
  return n < 1 ? 1 : n;
}

template <int R>
KK3_FN void mla_combine_item(const StepArgs& a, int layer, int hh, int r0, int nr, unsigned char* sm, int ph = -1) {
  const Geo& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // the head's value rows (vd x kr bf16) are read in step 3: bring them into L2 while steps 1-2 run
  {
    const unsigned char* kv = reinterpret_cast<const unsigned char*>(
        lptr<bf16>(a, layer, KK3_MLA_KB) + ((size_t)hh * (g.nr + g.vd) + g.nr) * g.kr);
    const int lines = g.vd * g.kr * 2 / 128;
    for (int i = tid; i < lines; i += kThreads) asm volatile("prefetch.global.L2 [%0];" ::"l"(kv + (size_t)i * 128));
  }
  const bool stamp = ph >= 0 && hh == 0 && r0 == 0 && tid == 0;   // sub-phase stamps of one item
  if (stamp) sub_stamp(a, ph, 0);
  const bool* reset = reinterpret_cast<const bool*>(a.ptr[KK3_RESET]);
  const int stride = g.kr + 2;
  const size_t cstride = (size_t)g.hr * stride;
  bf16* lat = reinterpret_cast<bf16*>(sm);                                     // [nr][8][kCombRow]
  float* wgt = reinterpret_cast<float*>(sm + (size_t)kCombRows * 8 * kCombRow * 2);   // [nr][64]
  float* lw = wgt + kCombRows * 64;                                            // [nr][64] w_i * l_i
  float* inv = lw + kCombRows * 64;                                            // [nr]
  // 1. chunk weights: every lane loads its chunks' (m, l); L is summed in chunk order by lane 0
  for (int r = warp; r < nr; r += kWarps) {
    const int b = r0 + r, nck = mla_row_chunks(a, b);
    const float* base = a.s.mla_part + (((size_t)b * g.mla_chunks) * g.hr + hh) * stride;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    if (lane < nck) {
      m0 = ld_cg_f32(base + lane * cstride);
      l0 = ld_cg_f32(base + lane * cstride + 1);
    }
    if (lane + 32 < nck) {
      m1 = ld_cg_f32(base + (lane + 32) * cstride);
      l1 = ld_cg_f32(base + (lane + 32) * cstride + 1);
    }
    const float M = warp_max(fmaxf(m0, m1));
    const float w0 = (lane < nck && m0 != -INFINITY) ? expf(m0 - M) : 0.0f;
    const float w1 = (lane + 32 < nck && m1 != -INFINITY) ? expf(m1 - M) : 0.0f;
    wgt[r * 64 + lane] = w0;
    wgt[r * 64 + lane + 32] = w1;
    lw[r * 64 + lane] = w0 * l0;
    lw[r * 64 + lane + 32] = w1 * l1;
    __syncwarp();
    if (lane == 0) {
      float L = 0.0f;
      for (int i = 0; i < nck; ++i) L += lw[r * 64 + i];
      inv[r] = 1.0f / L;
    }
  }
  __syncthreads();
  if (stamp) sub_stamp(a, ph, 1);
  // 2. attended latent rows (thread = latent dim), 32 loads in flight per round (32 / R chunks of each of R
  // rows: the partials may sit in the other die's L2, ~2 us away); chunks past a row's count have weight 0
  // and are not read
  constexpr int CK = 32 / R;
  for (int cc = tid; cc < g.kr; cc += kThreads) {
    float acc[R];
    int nck[R];
    const float* src[R];
    int nmax = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      acc[r] = 0.0f;
      nck[r] = r < nr ? mla_row_chunks(a, r0 + r) : 0;
      nmax = nck[r] > nmax ? nck[r] : nmax;
      src[r] = a.s.mla_part + (((size_t)(r0 + (r < nr ? r : 0)) * g.mla_chunks) * g.hr + hh) * stride + 2 + cc;
    }
    for (int i0 = 0; i0 < nmax; i0 += CK) {
      float v[R][CK];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int k = 0; k < CK; ++k) v[r][k] = i0 + k < nck[r] ? ld_cg_f32(src[r] + (size_t)(i0 + k) * cstride) : 0.0f;
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int k = 0; k < CK; ++k)
          if (i0 + k < nck[r]) acc[r] += wgt[r * 64 + i0 + k] * v[r][k];
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r >= nr) break;
      const bf16 lv = f2bf(acc[r] * inv[r]);
      lat[(r * 8 + (cc >> 6)) * kCombRow + (cc & 63)] = lv;
      // the attended latent (kimi.py:280) replaces the absorbed query in scratch, for diagnostics
      a.s.absorbed[(((size_t)(r0 + r)) * g.hr + hh) * g.kr + cc] = lv;
    }
  }
  __syncthreads();
  if (stamp) sub_stamp(a, ph, 2);
  // 3. value projection: two passes of 64 output dims, thread = (dim, 64-dim part of the latent)
  const int t = tid & 7;
  for (int pass = 0; pass < 2; ++pass) {
    const int dv = pass * 64 + (tid >> 3);
    __nv_bfloat162 w[8][4];   // this thread's 64 weights as bf16 pairs
    {
      const bf16* row = lptr<bf16>(a, layer, KK3_MLA_KB) + ((size_t)hh * (g.nr + g.vd) + g.nr + dv) * g.kr + t * 64;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uint4 u = *reinterpret_cast<const uint4*>(row + e * 8);
        w[e][0] = *reinterpret_cast<__nv_bfloat162*>(&u.x);
        w[e][1] = *reinterpret_cast<__nv_bfloat162*>(&u.y);
        w[e][2] = *reinterpret_cast<__nv_bfloat162*>(&u.z);
        w[e][3] = *reinterpret_cast<__nv_bfloat162*>(&u.w);
      }
    }
    for (int r = 0; r < nr; ++r) {
      float acc = 0.0f;
      const bf16* lr = lat + (r * 8 + t) * kCombRow;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint4 l4 = *reinterpret_cast<const uint4*>(lr + e * 8);
        const __nv_bfloat162* lv = reinterpret_cast<const __nv_bfloat162*>(&l4);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 wf = __bfloat1622float2(w[e][q]), lf = __bfloat1622float2(lv[q]);
          acc += wf.x * lf.x;
          acc += wf.y * lf.y;
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      if (t == 0) {
        const int b = r0 + r;
        const float o = round_bf(acc);
        const float gt = round_bf(sigmoidf_(bf2f(a.s.og[(size_t)b * g.hr * g.vd + hh * g.vd + dv])));
        a.s.attn_in[(size_t)b * g.hr * g.vd + hh * g.vd + dv] = f2bf(o * gt);
      }
    }
    if (stamp) sub_stamp(a, ph, 3 + pass);
  }
  __syncthreads();
}

// ------------------------------------------------------------------------------------------------
// Routing (kimi.py:308-316), done by every CTA at the start of the expert gate/up phase: warp w routes batch
// rows w, w + 16, ... (sigmoid scores + bias held 32 per lane, top-k with the lowest index winning ties,
// weights renormalised over the unbiased scores, ids sorted ascending), then the CTA groups the (row, slot)
// pairs by expert into chunks of <= 8 pairs for the MXFP4 phases. Every CTA computes the same tables and
// writes them (identical values), so the experts start without a grid barrier of their own.

// shared memory of the routing step: the selected ids [kMaxBatch * kMaxTopk] at 0; the grouping's per-expert
// row masks and offsets and its scan totals after them (< 32 KB); then each warp's scores and the router
// bias, lane-major [lane][kRouteStride] with a padded stride
constexpr int kRouteStride = 36;   // u32 words per lane: up to 32 keys (E <= 1024) plus padding
constexpr size_t kRouteKeyOff = 32 * 1024;
constexpr size_t kRouteBiasOff = kRouteKeyOff + (size_t)kWarps * 32 * kRouteStride * 4;
constexpr size_t kRouteSmem = kRouteBiasOff + (size_t)32 * kRouteStride * 4;
static_assert((size_t)kMaxBatch * kMaxTopk * 4 + (size_t)kMaxExperts * 16 + 2 * kWarps * 4 <= kRouteKeyOff,
              "routing tables overlap the keys");

KK3_DEV unsigned warp_excl_scan(unsigned v) {
  const int lane = threadIdx.x & 31;
  unsigned x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += t;
  }
  return x - v;
}

// group the pairs whose expert ids are in smem[0, B*K) by expert and write the pair and chunk tables. Every
// CTA writes these tables, so the order must not depend on thread timing: a row holds an expert at most once,
// so the pairs of expert e are placed in batch-row order through a 64-bit mask of the rows that chose e.
KK3_DEV void route_group_pairs(const StepArgs& a, unsigned char* smem) {
  const Geo& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = g.K;   // <= 32: pair (b, j) is handled by lane j of a warp
  const int* ids = reinterpret_cast<const int*>(smem);                                     // [B*K]
  unsigned long long* rows = reinterpret_cast<unsigned long long*>(smem + kMaxBatch * kMaxTopk * 4);   // [E]
  int* off = reinterpret_cast<int*>(rows + kMaxExperts);   // [E] first pair of each expert
  int* coff = off + kMaxExperts;                           // [E] first chunk of each expert
  int* wtot = coff + kMaxExperts;                          // [2][kWarps]
  // cold code (once per layer): compact loops, no divisions
#pragma unroll 1
  for (int e = tid; e < g.E; e += kThreads) rows[e] = 0ull;
  __syncthreads();
#pragma unroll 1
  for (int b = warp; b < g.B; b += kWarps)
    if (lane < K) atomicOr(&rows[ids[b * K + lane]], 1ull << b);
  __syncthreads();
  // exclusive scans over experts of pair counts and chunk counts: warp w scans experts [64w, 64w + 64)
  // (two per lane), then the warp totals are scanned (E <= 1024 = kWarps * 64)
  {
    const int ea = warp * 64 + 2 * lane, eb = ea + 1;
    const int na = ea < g.E ? __popcll(rows[ea]) : 0, nb = eb < g.E ? __popcll(rows[eb]) : 0;
    const int ca = (na + 7) >> 3, cb = (nb + 7) >> 3;
    const int pa = warp_excl_scan((unsigned)(na + nb)), pc = warp_excl_scan((unsigned)(ca + cb));
    if (lane == 31) {
      wtot[warp] = pa + na + nb;
      wtot[kWarps + warp] = pc + ca + cb;
    }
    __syncthreads();
    // exclusive prefix of the warp totals: lane w < kWarps holds warp w's totals, scanned with shuffles
    int tp = lane < kWarps ? wtot[lane] : 0, tc = lane < kWarps ? wtot[kWarps + lane] : 0;
#pragma unroll
    for (int o = 1; o < kWarps; o <<= 1) {
      const int up = __shfl_up_sync(0xffffffffu, tp, o), uc = __shfl_up_sync(0xffffffffu, tc, o);
      if (lane >= o) {
        tp += up;
        tc += uc;
      }
    }
    const int base = warp > 0 ? __shfl_sync(0xffffffffu, tp, warp - 1) : 0;
    const int cbase = warp > 0 ? __shfl_sync(0xffffffffu, tc, warp - 1) : 0;
    const int ctotal = __shfl_sync(0xffffffffu, tc, kWarps - 1);
    if (ea < g.E) {
      off[ea] = base + pa;
      coff[ea] = cbase + pc;
    }
    if (eb < g.E) {
      off[eb] = base + pa + na;
      coff[eb] = cbase + pc + ca;
    }
    if (tid == 0) a.s.chunk_info[0] = ctotal;
  }
  __syncthreads();
#pragma unroll 1
  for (int b = warp; b < g.B; b += kWarps) {
    if (lane < K) {
      const int e = ids[b * K + lane];
      const int pos = off[e] + __popcll(rows[e] & ((1ull << b) - 1ull));
      a.s.pair_row[pos] = b;
      a.s.pair_slot[pos] = lane;
    }
  }
#pragma unroll 1
  for (int e = tid; e < g.E; e += kThreads) {
    const int n = __popcll(rows[e]);
#pragma unroll 1
    for (int q = 0; q * 8 < n; ++q) {
      int* ci = a.s.chunk_info + 1 + (coff[e] + q) * 3;
      ci[0] = e;
      ci[1] = off[e] + q * 8;
      ci[2] = n - q * 8 < 8 ? n - q * 8 : 8;
    }
  }
}

// order-preserving 32-bit key of a routing value (a larger value has a larger key). NaN counts as -inf and
// -0 is keyed as +0, so values that compare equal have equal keys; absent entries get key 0, below them all.
KK3_DEV unsigned route_key(float x) {
  x = x != x ? -INFINITY : x;
  x = x == 0.0f ? 0.0f : x;
  const unsigned u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}


KK3_DEV unsigned warp_sum_u32(unsigned v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Warp w routes batch rows w, w + 16, ...; lane l holds the keys of experts [l * n, l * n + n) (n = E / 32
// rounded up) in registers, computed from a shared-memory staging copy (cp.async) of the row's scores and of
// the bias, read 16 bytes at a time. The K-th largest key T is found by bisection: the bits above the
// highest bit in which the largest and the smallest key differ are common to all keys, and the remaining bits
// are resolved two per round (three probes counted together) with warp-wide counts, stopping as soon as
// exactly K keys are >= the chosen probe. Every expert above T is taken, and of those equal to T the lowest
// indices (torch.topk's order as the reference uses it: value descending, then index ascending); lane-order
// prefix sums place the ids in ascending order.
KK3_FN void route_cta(const StepArgs& a, int layer, unsigned char* smem, int ph = -1) {
  const Geo& g = a.g;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = g.K, E = g.E;
  constexpr int kPer = kRouteStride - 4;   // 32 keys per lane at most (E <= 1024)
  const int nper = (E + 31) >> 5, e0 = lane * nper;
  const int nlive = E - e0 < 0 ? 0 : (E - e0 < nper ? E - e0 : nper);   // this lane's real experts
  int* ids = reinterpret_cast<int*>(smem);   // [B*K] sorted per row
  // bias and each warp's scores: linear ([e], lane l's run at l * n) when n % 4 == 0 and E % 4 == 0, so that
  // the staging copies are coalesced 16-byte pieces and each lane reads its run 16 bytes at a time (a lane
  // stride of n words, a multiple of 4 but not of 8, is bank-conflict free); else lane-major rows
  // [lane][kRouteStride] filled with 4-byte copies
  const bool lin = (nper & 3) == 0 && (E & 3) == 0;
  const int lstride = lin ? nper : kRouteStride;
  float* bias_w = reinterpret_cast<float*>(smem + kRouteBiasOff);
  float* bias_l = bias_w + lane * lstride;
  float* sc_w = reinterpret_cast<float*>(smem + kRouteKeyOff) + (size_t)warp * 32 * kRouteStride;
  float* sc_l = sc_w + lane * lstride;
  const float* bias = lptr<float>(a, layer, KK3_MOE_ROUTER_BIAS);
  long long* out_ids = gout<long long>(a, KK3_OUT_EXPERT_IDS) + (size_t)layer * g.B * K;
  const bool stamp = ph >= 0 && blockIdx.x == 0 && tid == 0;
  auto stage_row = [&](int b) {
    if (lin) {
      const float* sc = a.s.scores + (size_t)b * E;
#pragma unroll 1
      for (int q = lane; q < (E >> 2); q += 32) cp_async16(sc_w + 4 * q, sc + 4 * q);
    } else {
      const float* sc = a.s.scores + (size_t)b * E + e0;
#pragma unroll 1
      for (int i = 0; i < nlive; ++i) cp_async4_ca(sc_l + i, sc + i);
    }
  };
  if (lin) {
#pragma unroll 1
    for (int q = tid; q < (E >> 2); q += kThreads) cp_async16(bias_w + 4 * q, bias + 4 * q);
  } else if (warp == 0) {
#pragma unroll 1
    for (int i = 0; i < nlive; ++i) cp_async4_ca(bias_l + i, bias + e0 + i);
  }
  if (warp < g.B) stage_row(warp);
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  if (stamp) sub_stamp(a, ph, 9);
#pragma unroll 1
  for (int b = warp; b < g.B; b += kWarps) {
    if (b != warp) {
      __syncwarp();   // every lane is done with the previous row (linear layout: lanes read each other's copies)
      stage_row(b);
      cp_async_commit();
      cp_async_wait_all();
      __syncwarp();
    }
    // keys; absent experts and padding get key 0, below every real key
    unsigned key[kPer];
    unsigned kmax = 0u, kmin = 0xffffffffu;
#pragma unroll
    for (int q = 0; q < kPer / 4; ++q) {
      const float4 sv = reinterpret_cast<const float4*>(sc_l)[q], bv = reinterpret_cast<const float4*>(bias_l)[q];
      const float x[4] = {sv.x + bv.x, sv.y + bv.y, sv.z + bv.z, sv.w + bv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = 4 * q + j;
        key[i] = i < nlive ? route_key(x[j]) : 0u;
        if (i < nlive) {
          kmax = key[i] > kmax ? key[i] : kmax;
          kmin = key[i] < kmin ? key[i] : kmin;
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned x = __shfl_xor_sync(0xffffffffu, kmax, o), y = __shfl_xor_sync(0xffffffffu, kmin, o);
      kmax = x > kmax ? x : kmax;
      kmin = y < kmin ? y : kmin;
    }
    if (stamp && b == 0) sub_stamp(a, ph, 10);
    int bit = 31 - __clz(kmax ^ kmin);   // -1 when every key is equal
    unsigned T = bit < 0 ? kmax : (bit >= 31 ? 0u : (kmax & ~((2u << bit) - 1u)));
    bool done = false;
#pragma unroll 1
    for (; bit >= 1 && !done; bit -= 2) {
      // probes T|hi, T|lo|... : p1 = T + lo, p2 = T + hi, p3 = T + hi + lo (lo = bit - 1, hi = bit)
      const unsigned hi = 1u << bit, lo = 1u << (bit - 1);
      const unsigned p1 = T | lo, p2 = T | hi, p3 = T | hi | lo;
      unsigned n1 = 0, n2 = 0, n3 = 0;
#pragma unroll
      for (int i = 0; i < kPer; ++i) {
        n1 += key[i] >= p1 ? 1u : 0u;
        n2 += key[i] >= p2 ? 1u : 0u;
        n3 += key[i] >= p3 ? 1u : 0u;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        n1 += __shfl_xor_sync(0xffffffffu, n1, o);
        n2 += __shfl_xor_sync(0xffffffffu, n2, o);
        n3 += __shfl_xor_sync(0xffffffffu, n3, o);
      }
      const unsigned k = (unsigned)K;
      if (n3 >= k) { T = p3; done = n3 == k; }
      else if (n2 >= k) { T = p2; done = n2 == k; }
      else if (n1 >= k) { T = p1; done = n1 == k; }
    }
    if (!done && bit == 0) {   // an odd number of bits: the last one alone
      const unsigned p = T | 1u;
      unsigned n = 0;
#pragma unroll
      for (int i = 0; i < kPer; ++i) n += key[i] >= p ? 1u : 0u;
      n = warp_sum_u32(n);
      if (n >= (unsigned)K) T = p;
    }
    if (stamp && b == 0) sub_stamp(a, ph, 12);
    // take every key above T and, in index order, the first K - #(above) keys equal to T
    unsigned gt = 0, eq = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      gt += key[i] > T ? 1u : 0u;
      eq += key[i] == T ? 1u : 0u;
    }
    const unsigned need = (unsigned)K - warp_sum_u32(gt);
    const unsigned tie0 = warp_excl_scan(eq);
    unsigned ties = tie0 < need ? (need - tie0 < eq ? need - tie0 : eq) : 0u;   // ties this lane takes
    unsigned pos = warp_excl_scan(gt + ties);
    int* row_ids = ids + b * K;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      bool take = key[i] > T;
      if (key[i] == T && ties > 0) {
        take = true;
        --ties;
      }
      if (take) {
        if (pos < (unsigned)K) row_ids[pos] = e0 + i;
        ++pos;
      }
    }
    __syncwarp();
    if (stamp && b == 0) sub_stamp(a, ph, 13);
    // weights: the unbiased scores of the chosen experts, from the staged row
    int e = lane < K ? row_ids[lane] : 0;
    e = e < 0 ? 0 : (e >= E ? E - 1 : e);
    const float w = lane < K ? sc_w[lin ? e : (e / nper) * kRouteStride + e % nper] : 0.0f;
    const float wsum = warp_sum(w);
    if (lane < K) {
      row_ids[lane] = e;
      a.s.route_ids[b * K + lane] = e;
      a.s.route_w[b * K + lane] = w / (wsum + 1e-20f);
      out_ids[(size_t)b * K + lane] = (long long)e;
    }
    __syncwarp();
  }
  __syncthreads();
  if (stamp) sub_stamp(a, ph, 14);
  route_group_pairs(a, smem);
  __syncthreads();
  if (stamp) sub_stamp(a, ph, 15);
}

}  // namespace kk3
