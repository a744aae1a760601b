// Checker of the tensor-core expert engine (kk3_tc_experts.cuh) against the decode step's mma.sync engine
// (run_experts, kk3_gemv.cuh) on one expert geometry (batch 8, 16 of 896 experts per row, latent 3584, expert
// intermediate 384 for a TP8 rank by default), random MXFP4 codes and E8M0 scales, bf16-valued latent rows.
//
// Both engines run gate/up (kimi.py:317-319: situ(gate, up) per pair) and then down (:320-323) on the same
// routed batch. Prints one JSON line: the fraction of bit-identical activations and slot outputs, the largest
// difference relative to the largest value, each phase's best time over `reps` launches with the L2 flushed
// before each, and the device error word. Routing tables are built on the host exactly as the step's routing
// groups pairs (by expert, chunks of <= 8 pairs); experts are folded into `distinct_experts` ones to bound
// memory.
//
//     kk3_tc_check [reps] [expert_intermediate] [distinct_experts]
//     (intermediate 384: one TP8 rank, the default; 3072: TP1. Distinct experts: 160 by default, at most 896)
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <vector>

#include "kk3_tc_experts.cuh"

using namespace kk3;

template <int MT>
__global__ void __launch_bounds__(512, 1) mma_engine(const __grid_constant__ StepArgs a, const __grid_constant__ ExpertPhase ph) {
  if (threadIdx.x == 0) kk3_cur_phase = -1;
  __syncthreads();
  run_experts<MT>(a, ph);
}
template <int MT>
__global__ void __launch_bounds__(512, 1) tc_engine(const __grid_constant__ StepArgs a, const __grid_constant__ TcPhase ph, int smem) {
  run_experts_tc<MT>(a, ph, smem);
}
__global__ void __launch_bounds__(512, 1) tc_quant(const __grid_constant__ StepArgs a, const __half* x, int K, int npairs,
                                                   int atoms, uint8_t* img, uint8_t* sfb) {
  tc_quant_pairs(a, x, K, npairs, atoms, img, sfb);
}

#define CK(x)                                                                       \
  do {                                                                              \
    cudaError_t e_ = (x);                                                           \
    if (e_ != cudaSuccess) {                                                        \
      printf("{\"error\": \"%s: %s\"}\n", #x, cudaGetErrorString(e_));             \
      return 1;                                                                     \
    }                                                                               \
  } while (0)

static PFN_cuTensorMapEncodeTiled_v12000 g_encode;

// codes of E experts [E, rows, K/2] as 4-bit elements: 256-row x 128-k boxes, 128-byte swizzle
static int make_map(CUtensorMap* m, void* base, int K, int rows, int E) {
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)rows, (cuuint64_t)E};
  cuuint64_t strides[2] = {(cuuint64_t)K / 2, (cuuint64_t)rows * K / 2};
  cuuint32_t box[3] = {128, kTcRows, 1}, es[3] = {1, 1, 1};
  return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : 1;
}
static float h2f(uint16_t h) {
  __half x;
  memcpy(&x, &h, 2);
  return __half2float(x);
}
static float bfh2f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

int main(int argc, char** argv) {
  const int reps = argc > 1 ? atoi(argv[1]) : 3;
  const int B = 8, E = 896, K = 16, lh = 3584;
  const int inter = argc > 2 ? atoi(argv[2]) : 384, nuse = argc > 3 ? atoi(argv[3]) : 160;
  if (inter <= 0 || inter % 128 != 0 || nuse < 1 || nuse > E) {
    printf("{\"error\": \"expert_intermediate must be a positive multiple of 128, distinct_experts in [1, 896]\"}\n");
    return 1;
  }
  int dev = 0, sms = 0;
  CK(cudaGetDevice(&dev));
  CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  cudaDriverEntryPointQueryResult qr;
  CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", (void**)&g_encode, cudaEnableDefault, &qr));
  static StepArgs a;
  memset(&a, 0, sizeof(a));
  a.g.B = B; a.g.E = E; a.g.K = K; a.g.lh = lh; a.g.inter = inter; a.g.L = 1; a.g.timeout_ns = 200000000ll;

  // routing: K distinct experts per row; expert 5 shared by four rows so that one chunk holds several pairs
  std::mt19937 rng(11);
  std::vector<int> ids(B * K);
  for (int b = 0; b < B; ++b) {
    std::vector<int> all(E);
    for (int e = 0; e < E; ++e) all[e] = e;
    for (int j = 0; j < K; ++j) std::swap(all[j], all[j + rng() % (E - j)]);
    std::sort(all.begin(), all.begin() + K);
    for (int j = 0; j < K; ++j) ids[b * K + j] = all[j];
  }
  for (int b = 0; b < B; b += 2) ids[b * K] = 5;
  std::vector<int> pair_row, pair_slot, chunk(1, 0);
  for (int e = 0; e < E; ++e) {
    std::vector<std::pair<int, int>> ps;
    for (int b = 0; b < B; ++b)
      for (int j = 0; j < K; ++j)
        if (ids[b * K + j] == e) ps.push_back({b, j});
    for (size_t q = 0; q < ps.size(); q += 8) {
      chunk.push_back(e % nuse);
      chunk.push_back((int)pair_row.size());
      chunk.push_back((int)std::min<size_t>(8, ps.size() - q));
      for (size_t t = q; t < std::min(ps.size(), q + 8); ++t) {
        pair_row.push_back(ps[t].first);
        pair_slot.push_back(ps[t].second);
      }
      chunk[0]++;
    }
  }
  const int npairs = (int)pair_row.size(), nch = chunk[0];

  // weights and the latent rows
  const size_t ce = (size_t)inter * lh / 2, se = (size_t)inter * lh / 32;
  std::vector<uint8_t> hc(ce * nuse), hs(se * nuse);
  uint8_t* w[6];
  for (int i = 0; i < 6; ++i) {
    const size_t n = i < 3 ? ce * nuse : se * nuse;
    CK(cudaMalloc(&w[i], n));
    auto& h = i < 3 ? hc : hs;
    for (auto& c : h) c = i < 3 ? (uint8_t)(rng() & 0xff) : (uint8_t)(118 + rng() % 6);
    CK(cudaMemcpy(w[i], h.data(), n, cudaMemcpyHostToDevice));
  }
  uint8_t *gate = w[0], *up = w[1], *down = w[2], *gs = w[3], *us = w[4], *ds = w[5];
  std::vector<uint16_t> hlat(B * lh);
  std::normal_distribution<float> nd(0.f, 2.f);
  for (auto& v : hlat) {
    float f = nd(rng);
    uint32_t u;
    memcpy(&u, &f, 4);
    u = (u + 0x8000u) & 0xffff0000u;   // bf16-valued
    memcpy(&f, &u, 4);
    __half h = __float2half_rn(f);
    memcpy(&v, &h, 2);
  }
  int *d_chunk, *d_prow, *d_pslot, *d_cnt, *d_cnt2, *d_err;
  float *d_part, *d_part2;
  __half *d_lat, *d_act, *d_act2;
  bf16 *d_out, *d_out2;
  const size_t act_b = (size_t)B * K * inter * 2, out_b = (size_t)B * K * lh * 2;
  CK(cudaMalloc(&d_chunk, chunk.size() * 4)); CK(cudaMalloc(&d_prow, B * K * 4)); CK(cudaMalloc(&d_pslot, B * K * 4));
  CK(cudaMalloc(&d_cnt, 1 << 22)); CK(cudaMalloc(&d_cnt2, 1 << 22)); CK(cudaMalloc(&d_err, 64));
  CK(cudaMalloc(&d_part, 64 << 20)); CK(cudaMalloc(&d_part2, 16 << 20));
  CK(cudaMalloc(&d_lat, B * lh * 2)); CK(cudaMalloc(&d_act, act_b)); CK(cudaMalloc(&d_act2, act_b));
  CK(cudaMalloc(&d_out, out_b)); CK(cudaMalloc(&d_out2, out_b));
  CK(cudaMemset(d_cnt, 0, 1 << 22)); CK(cudaMemset(d_cnt2, 0, 1 << 22)); CK(cudaMemset(d_err, 0, 64));
  CK(cudaMemset(d_act, 0, act_b)); CK(cudaMemset(d_act2, 0, act_b)); CK(cudaMemset(d_out, 0, out_b)); CK(cudaMemset(d_out2, 0, out_b));
  CK(cudaMemcpy(d_lat, hlat.data(), hlat.size() * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(d_chunk, chunk.data(), chunk.size() * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(d_prow, pair_row.data(), npairs * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(d_pslot, pair_slot.data(), npairs * 4, cudaMemcpyHostToDevice));
  a.s.chunk_info = d_chunk; a.s.pair_row = d_prow; a.s.pair_slot = d_pslot; a.s.fix_cnt = d_cnt; a.s.fix_part = d_part;
  a.s.latent_p = d_lat; a.s.act_p = d_act; a.s.out_slot = d_out; a.s.err = d_err; a.s.err_host = d_err + 4;

  // activation images of the tensor-core engine (latent per pair, then the activations)
  const int atoms = (B * K + 7) / 8;
  uint8_t *limg, *lsfb, *aimg, *asfb;
  const size_t limg_b = (size_t)(lh / 128) * atoms * 2048, lsfb_b = (size_t)(lh / 128) * atoms * 256;
  const size_t aimg_b = (size_t)(inter / 128) * atoms * 2048, asfb_b = (size_t)(inter / 128) * atoms * 256;
  CK(cudaMalloc(&limg, limg_b)); CK(cudaMalloc(&lsfb, lsfb_b)); CK(cudaMalloc(&aimg, aimg_b)); CK(cudaMalloc(&asfb, asfb_b));
  CK(cudaMemset(aimg, 0, aimg_b)); CK(cudaMemset(asfb, 127, asfb_b));
  CUtensorMap hm[3];
  if (make_map(&hm[0], gate, lh, inter, nuse) || make_map(&hm[1], up, lh, inter, nuse) || make_map(&hm[2], down, inter, lh, nuse)) {
    printf("{\"error\": \"cuTensorMapEncodeTiled failed\"}\n");
    return 1;
  }
  CUtensorMap* dm;
  CK(cudaMalloc(&dm, sizeof(hm)));
  CK(cudaMemcpy(dm, hm, sizeof(hm), cudaMemcpyHostToDevice));

  ExpertPhase gu{}, dn{};
  gu.codes[0] = gate; gu.codes[1] = up; gu.scales[0] = gs; gu.scales[1] = us;
  gu.rows = inter; gu.K = lh; gu.tiles = inter / 16; gu.ksteps = lh / 64; gu.expert_codes = ce; gu.expert_scales = se;
  dn.codes[0] = dn.codes[1] = down; dn.scales[0] = dn.scales[1] = ds;
  dn.rows = lh; dn.K = inter; dn.tiles = lh / 16; dn.ksteps = inter / 64; dn.expert_codes = ce; dn.expert_scales = se;
  TcPhase tg{}, td{};
  tg.map[0] = dm; tg.map[1] = dm + 1; tg.scales[0] = gs; tg.scales[1] = us;
  tg.rows = inter; tg.K = lh; tg.tiles = (inter + kTcRows - 1) / kTcRows; tg.ksteps = lh / 128; tg.expert_scales = se;
  tg.bimg = limg; tg.bsfb = lsfb; tg.atoms = atoms; tg.part = d_part2; tg.cnt = d_cnt2;
  tg.oimg = aimg; tg.osfb = asfb; tg.act_dbg = d_act2;
  td.map[0] = td.map[1] = dm + 2; td.scales[0] = td.scales[1] = ds;
  td.rows = lh; td.K = inter; td.tiles = (lh + kTcRows - 1) / kTcRows; td.ksteps = inter / 128; td.expert_scales = se;
  td.bimg = aimg; td.bsfb = asfb; td.atoms = atoms; td.part = d_part2; td.cnt = d_cnt2;
  StepArgs a2 = a;
  a2.s.out_slot = d_out2;

  const int sm_mma = kExpSmem, sm_tc = 3 * tc_stage_bytes<2>();
  CK(cudaFuncSetAttribute(mma_engine<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm_mma));
  CK(cudaFuncSetAttribute(mma_engine<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm_mma));
  CK(cudaFuncSetAttribute(tc_engine<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm_tc));
  CK(cudaFuncSetAttribute(tc_engine<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, sm_tc));
  auto launch = [&](int which) {
    switch (which) {
      case 0: mma_engine<2><<<sms, 512, sm_mma>>>(a, gu); break;
      case 1: mma_engine<1><<<sms, 512, sm_mma>>>(a, dn); break;
      case 2: tc_quant<<<sms, 512>>>(a, d_lat, lh, npairs, atoms, limg, lsfb); break;
      case 3: tc_engine<2><<<sms, 512, sm_tc>>>(a, tg, sm_tc); break;
      default: tc_engine<1><<<sms, 512, sm_tc>>>(a2, td, sm_tc); break;
    }
  };
  for (int which = 0; which < 5; ++which) {
    launch(which);
    CK(cudaDeviceSynchronize());
  }
  int herr = 0;
  CK(cudaMemcpy(&herr, d_err, 4, cudaMemcpyDeviceToHost));

  // compare: activations of the gate/up phase, then the down projection's slot outputs
  std::vector<uint16_t> x1((size_t)npairs * inter), x2(x1.size());
  CK(cudaMemcpy(x1.data(), d_act, x1.size() * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(x2.data(), d_act2, x2.size() * 2, cudaMemcpyDeviceToHost));
  double amax = 0, adiff = 0;
  size_t asame = 0;
  for (size_t i = 0; i < x1.size(); ++i) {
    const float u = h2f(x1[i]), v = h2f(x2[i]);
    amax = std::max(amax, (double)fabsf(u));
    adiff = std::max(adiff, (double)fabsf(u - v));
    asame += x1[i] == x2[i];
  }
  std::vector<uint16_t> o1((size_t)B * K * lh), o2(o1.size());
  CK(cudaMemcpy(o1.data(), d_out, o1.size() * 2, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(o2.data(), d_out2, o2.size() * 2, cudaMemcpyDeviceToHost));
  double omax = 0, odiff = 0;
  size_t osame = 0;
  for (size_t i = 0; i < o1.size(); ++i) {
    const float u = bfh2f(o1[i]), v = bfh2f(o2[i]);
    omax = std::max(omax, (double)fabsf(u));
    odiff = std::max(odiff, (double)fabsf(u - v));
    osame += o1[i] == o2[i];
  }

  // timing: best of `reps` launches, L2 flushed (1 GiB written) before each
  float* flush;
  CK(cudaMalloc(&flush, 1 << 30));
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  float best[5];
  for (int which = 0; which < 5; ++which) {
    best[which] = 1e9f;
    for (int it = 0; it < reps; ++it) {
      CK(cudaMemset(flush, it, 1 << 30));
      CK(cudaEventRecord(e0));
      launch(which);
      CK(cudaEventRecord(e1));
      CK(cudaEventSynchronize(e1));
      float ms;
      CK(cudaEventElapsedTime(&ms, e0, e1));
      best[which] = std::min(best[which], ms * 1000.0f);
    }
  }
  CK(cudaMemcpy(&herr, d_err, 4, cudaMemcpyDeviceToHost));
  const double gu_bytes = (double)nch * 2 * (ce + se), dn_bytes = (double)nch * (ce + se);
  printf("{\"chunks\": %d, \"pairs\": %d, \"act_identical\": %.6f, \"act_max_rel_diff\": %.3g, "
         "\"out_identical\": %.6f, \"out_max_rel_diff\": %.3g, \"mma_gate_up_us\": %.2f, \"mma_down_us\": %.2f, "
         "\"tc_quant_us\": %.2f, \"tc_gate_up_us\": %.2f, \"tc_down_us\": %.2f, \"gate_up_mb\": %.1f, "
         "\"down_mb\": %.1f, \"error_word\": %d}\n",
         nch, npairs, (double)asame / x1.size(), adiff / (amax > 0 ? amax : 1), (double)osame / o1.size(),
         odiff / (omax > 0 ? omax : 1), best[0], best[1], best[2], best[3], best[4], gu_bytes / 1e6, dn_bytes / 1e6, herr);
  return herr != 0;
}
