// kk3_host.cu - the C ABI declared in include/kk3.h: context set-up, peer mapping, launch, status.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "kk3_phases.cuh"

namespace kk3 {
// one instantiation per batch tile count, each in its own translation unit (kk3_kernel_nt*.cu)
#define KK3_DECL(n)                                                  \
  cudaError_t prepare_nt##n(size_t smem, int* occupancy);           \
  cudaError_t launch_nt##n(const StepArgs* args, int grid, size_t smem, cudaStream_t stream);
KK3_DECL(1)
KK3_DECL(2)
KK3_DECL(4)
KK3_DECL(8)
#undef KK3_DECL

static cudaError_t prepare_kernel(int nt, size_t smem, int* occ) {
  switch (nt) {
    case 1: return prepare_nt1(smem, occ);
    case 2: return prepare_nt2(smem, occ);
    case 4: return prepare_nt4(smem, occ);
    default: return prepare_nt8(smem, occ);
  }
}
static cudaError_t launch_kernel(int nt, const StepArgs* a, int grid, size_t smem, cudaStream_t st) {
  switch (nt) {
    case 1: return launch_nt1(a, grid, smem, st);
    case 2: return launch_nt2(a, grid, smem, st);
    case 4: return launch_nt4(a, grid, smem, st);
    default: return launch_nt8(a, grid, smem, st);
  }
}
}  // namespace kk3

using namespace kk3;

struct kk3_ctx {
  kk3_config cfg;
  Geo g;
  Scratch s;
  Comm comm;
  int sms = 0, grid = 0, nt = 1;
  size_t smem = 0;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  void* comm_local = nullptr;
  size_t comm_bytes = 0;
  void* peer_open[kMaxTp] = {};
  int* err_host = nullptr;
  int* err_dev = nullptr;
  int* trace_host = nullptr;   // mapped progress words (fault localisation): [2][1024] per CTA, [4096] per warp
  int* trace_dev = nullptr;
  int trace = 0;
  unsigned epoch = 0;
  int failed = 0;
  int peers_open = 0;
  int comm_mode = kCommPeer;
  int gemv_engine = kGemvAuto;
  StepArgs* args = nullptr;
  size_t buf_bytes[KK3_BUF_COUNT] = {};
  void* buf_ptr[KK3_BUF_COUNT] = {};
};

// MLA attention work split: heads in groups of at most four 16-row tiles (the accumulators of a group stay
// in registers), and each batch row's attended positions in chunks so that rows x chunks x groups items fill
// one wave of the grid.
static void plan_mla(Geo& g, int grid) {
  const int tiles = (g.hr + 15) / 16;
  g.mla_groups = (tiles + 3) / 4;
  g.mla_mt = (tiles + g.mla_groups - 1) / g.mla_groups;
  int chunks = grid / (g.B * g.mla_groups);
  chunks = chunks < 1 ? 1 : (chunks > 64 ? 64 : chunks);
  int len = (g.ctx + 1 + chunks - 1) / chunks;
  len = (len + kMlaPos - 1) / kMlaPos * kMlaPos;
  g.mla_chunk_len = len;
  g.mla_chunks = (g.ctx + 1 + len - 1) / len;
}

static int cuda_fail(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KK3_OK;
  fprintf(stderr, "kk3: %s failed: %s\n", what, cudaGetErrorString(e));
  return KK3_ERR_CUDA;
}
#define KK3_CUDA(call)                                 \
  do {                                                 \
    int rc_ = cuda_fail((call), #call);                \
    if (rc_ != KK3_OK) return rc_;                     \
  } while (0)

extern "C" int kk3_table_size(const kk3_config* cfg) {
  if (!cfg || cfg->layers < 1) return KK3_ERR_ARG;
  return KK3_GLOBAL_SLOTS + cfg->layers * KK3_LAYER_SLOTS;
}

extern "C" const char* kk3_error_string(int code) {
  switch (code) {
    case KK3_OK: return "ok";
    case KK3_ERR_ARG: return "bad argument or pointer table";
    case KK3_ERR_UNSUPPORTED: return "geometry not supported by the sm_100a kernels";
    case KK3_ERR_CUDA: return "CUDA runtime call failed";
    case KK3_ERR_TIMEOUT: return "in-kernel wait exceeded its bound (a peer or CTA never arrived)";
    case KK3_ERR_DEVICE: return "in-kernel consistency check failed";
    case KK3_ERR_PEERS: return "tensor-parallel peers are not open";
    case KK3_ERR_FAILED: return "context failed earlier; rebuild it";
    case KK3_ERR_TOO_LARGE: return "geometry needs more scratch than kk3_step_noalloc's static 32 MiB; use kk3_init";
    default: return "unknown kk3 error";
  }
}

static int validate(const kk3_config* c) {
  if (!c) return KK3_ERR_ARG;
  const bool ok =
      c->layers >= 1 && c->layers <= 96 && c->batch >= 1 && c->batch <= kMaxBatch && c->head_dim == 128 &&
      c->qk_nope_dim == 128 && c->v_head_dim == 128 && c->qk_rope_dim == 64 && c->kv_lora_rank == 512 &&
      c->conv_kernel == 4 && c->topk >= 1 && c->topk <= kMaxTopk && c->experts >= c->topk &&
      c->experts <= kMaxExperts && c->heads >= 1 && c->heads <= 96 && c->tp >= 1 && c->tp <= kMaxTp &&
      c->rank >= 0 && c->rank < c->tp && c->hidden % 64 == 0 && c->hidden <= 8192 && c->latent_hidden % 64 == 0 &&
      c->latent_hidden <= 8192 && c->q_lora_rank % 64 == 0 && c->inter_shard % 64 == 0 && c->inter_shard > 0 &&
      c->dense_inter_shard % 64 == 0 && c->shared_inter_shard % 64 == 0 && c->vocab_shard >= 1 &&
      c->context >= 1 && c->attn_res_block_size >= 1 && c->first_dense >= 0 &&
      (c->layers + c->attn_res_block_size - 1) / c->attn_res_block_size <= kMaxBlocks - 1 &&
      (long long)c->heads * 128 % 64 == 0 && (long long)c->vocab_shard * c->batch < (1ll << 31) &&
      // MoE layers: the expert engine walks 128-k unit pairs and copies scales in 16-byte pieces, either a
      // 16-byte window per row (K % 512 == 0) or the tile's whole scale block (gate/up: K = latent_hidden
      // <= 512; down: K = inter_shard <= 1024)
      (c->layers <= c->first_dense ||
       (c->latent_hidden % 128 == 0 && c->inter_shard % 128 == 0 &&
        (c->latent_hidden % 512 == 0 || c->latent_hidden <= 512) &&
        (c->inter_shard % 512 == 0 || c->inter_shard <= 1024)));
  return ok ? KK3_OK : KK3_ERR_UNSUPPORTED;
}

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// One planner for both entry points (kk3_init and kk3_step_noalloc): the geometry, the batch-tile class, the
// scratch layout and the dynamic shared memory of a step on a grid of `sms` CTAs. With base == nullptr only
// the sizes are computed. The scratch starts with the words that must be zero when a step begins (barrier,
// phase count, error word and its mirror, situ and stream-K counters, then the single-rank exchange block when
// `comm_inline`); `zero_bytes` covers them, the rest is written before it is read within every step.
// `profiling` adds the per-CTA barrier and per-warp engine stamps (context path only). `comm_inline` places a
// single rank's exchange buffer inside the scratch (the allocation-free path, tp == 1); otherwise the exchange
// buffer is a separate allocation, exported to peers over CUDA IPC.
struct StepPlan {
  Geo g;
  Scratch s;
  Comm comm;        // offsets always; comm.base[rank] only when comm_inline
  int nt;           // batch in 8-row n-tiles: 1, 2, 4 or 8
  size_t smem;      // dynamic shared memory of the step kernel
  size_t total;     // scratch bytes
  size_t zero;      // leading scratch bytes that must be zero at the start of a step
  size_t comm_bytes;
  size_t qkv_w;
};

static void plan_step(const kk3_config* cfg, int sms, unsigned char* base, bool profiling, bool comm_inline,
                      StepPlan* pl) {
  Geo& g = pl->g;
  memset(&g, 0, sizeof(g));
  g.L = cfg->layers; g.B = cfg->batch; g.h = cfg->hidden; g.lh = cfg->latent_hidden; g.inter = cfg->inter_shard;
  g.dinter = cfg->dense_inter_shard; g.sinter = cfg->shared_inter_shard; g.hr = cfg->heads; g.d = cfg->head_dim;
  g.qr = cfg->q_lora_rank; g.kr = cfg->kv_lora_rank; g.nr = cfg->qk_nope_dim; g.rd = cfg->qk_rope_dim;
  g.vd = cfg->v_head_dim; g.V = cfg->vocab_shard; g.E = cfg->experts; g.K = cfg->topk; g.ctx = cfg->context;
  g.conv = cfg->conv_kernel; g.bs = cfg->attn_res_block_size; g.first_dense = cfg->first_dense; g.tp = cfg->tp;
  g.rank = cfg->rank; g.qdim = g.hr * g.d;
  for (int l = 0; l < g.L; ++l) {
    if (((l + 1) % 4 == 0) || l == g.L - 1) ++g.nmla; else ++g.nkda;
  }
  g.nblk = (g.L + g.bs - 1) / g.bs;
  g.timeout_ns = cfg->timeout_ns > 0 ? cfg->timeout_ns : 10000000000ll;
  const int nt = g.B <= 8 ? 1 : (g.B <= 16 ? 2 : (g.B <= 32 ? 4 : 8));
  pl->nt = nt;
  g.bp = 8 * nt;
  plan_mla(g, sms);
  const long long gw = (long long)sms * kWarps;
  g.fix_bank = 2ll * gw * (2 * nt * 128);
  {
    long long tiles = 0;
    auto mx = [&](long long v) { tiles = v > tiles ? v : tiles; };
    mx((3ll * g.qdim + g.qdim + g.d + g.hr + 15 * 6) / 16 + 6);
    mx((long long)(g.qr + g.kr + g.rd + g.hr * g.vd) / 16 + 3);
    mx((long long)g.hr * (g.nr + g.rd) / 16 + 1);
    mx(g.h / 16 + 1);
    mx(2ll * ((g.dinter + 15) / 16) + 2);                                        // dense gate | up
    mx((long long)(g.E + 15) / 16 + (g.lh + 15) / 16 + 2ll * ((g.sinter + 15) / 16) + 4);   // MoE input pass
    mx((long long)(g.V + 15) / 16 + 1);
    mx((long long)g.B * g.K * ((g.inter > g.lh ? g.inter : g.lh) / 16));
    g.cnt_bank = (int)tiles;
  }
  const size_t B = g.B, tp = g.tp;
  const size_t qkv_w =
      (size_t)3 * g.qdim > (size_t)(g.qr + g.kr + g.rd) ? (size_t)3 * g.qdim : (size_t)(g.qr + g.kr + g.rd);
  pl->qkv_w = qkv_w;
  Scratch& s = pl->s;
  memset(&s, 0, sizeof(s));
  // situ pairs: tiles of the larger of the dense and shared-expert intermediates, 4 * NT floats per lane
  const size_t situ_tiles = (size_t)((g.dinter > g.sinter ? g.dinter : g.sinter) + 15) / 16 + 1;
  const size_t situ_floats = 2 * situ_tiles * 32 * 4 * (size_t)nt;
  // exchange buffer: flags [B][tp] u32, then two parity regions {att bf16 [tp][h/16][bp][16], exp f32
  // [tp][B][lh], shd bf16 [tp][h/16][bp][16], key u64 [tp][B]}; bp = 8 * nt, so that one 16-row GEMV tile of a
  // source is one contiguous block of the bf16 regions
  Comm& c = pl->comm;
  memset(&c, 0, sizeof(c));
  // flags: per-row flags [B][tp], then the push transport's per-chunk flags [tp][sms] (both start at zero)
  const size_t flag_bytes = align_up(B * tp * 4, 256) + align_up(tp * (size_t)sms * 4, 256);
  c.flag_off = 0;
  c.push_flag_off = (long long)align_up(B * tp * 4, 256);
  c.att_off = 0;
  size_t r = align_up(tp * (size_t)g.bp * g.h * 2, 256);
  c.exp_off = r;
  r += align_up(tp * B * g.lh * 4, 256);
  c.shd_off = r;
  r += align_up(tp * (size_t)g.bp * g.h * 2, 256);
  c.key_off = r;
  r += align_up(tp * B * 8, 256);
  c.region_bytes = r;
  c.data_off[0] = flag_bytes;
  c.data_off[1] = flag_bytes + r;
  pl->comm_bytes = flag_bytes + 2 * r;
  unsigned char* comm = nullptr;
  int* err_mirror = nullptr;
  struct Item { void** p; size_t bytes; };
  Item items[] = {
      // must be zero when a step begins
      {(void**)&s.bar, 64}, {(void**)&s.phase_count, 64}, {(void**)&s.err, 64}, {(void**)&err_mirror, 64},
      {(void**)&s.situ_cnt, situ_tiles * 4}, {(void**)&s.fix_cnt, (size_t)g.cnt_bank * 2 * 4},
      {(void**)&comm, comm_inline ? pl->comm_bytes : 0},
      // written before they are read within every step
      {(void**)&s.prefix, B * g.h * 2}, {(void**)&s.blocks, (size_t)g.nblk * B * g.h * 2},
      {(void**)&s.xa, B * g.h * 2}, {(void**)&s.xm, B * g.h * 2}, {(void**)&s.qkv, B * qkv_w * 2},
      {(void**)&s.og, B * (size_t)g.qdim * 2}, {(void**)&s.fa, B * g.d * 2}, {(void**)&s.beta, B * g.hr * 2},
      {(void**)&s.attn_in, B * (size_t)g.hr * g.vd * 2}, {(void**)&s.mla_qan, B * g.qr * 2},
      {(void**)&s.mla_q, B * (size_t)g.hr * (g.nr + g.rd) * 2}, {(void**)&s.absorbed, B * (size_t)g.hr * g.kr * 2},
      {(void**)&s.mla_part, B * (size_t)g.mla_chunks * g.hr * (g.kr + 2) * 4},
      {(void**)&s.dense_act, B * (size_t)(g.dinter > 0 ? g.dinter : 64) * 2}, {(void**)&s.scores, B * g.E * 4},
      {(void**)&s.latent, B * g.lh * 2}, {(void**)&s.latent_p, B * g.lh * 2},
      {(void**)&s.shared_act, B * (size_t)(g.sinter > 0 ? g.sinter : 64) * 2}, {(void**)&s.route_ids, B * g.K * 4},
      {(void**)&s.route_w, B * g.K * 4}, {(void**)&s.pair_row, B * g.K * 4}, {(void**)&s.pair_slot, B * g.K * 4},
      {(void**)&s.chunk_info, (1 + B * g.K * 3) * 4}, {(void**)&s.act_p, B * g.K * (size_t)g.inter * 2},
      {(void**)&s.out_slot, B * g.K * (size_t)g.lh * 2}, {(void**)&s.x3, B * g.lh * 2},
      {(void**)&s.shared_red, B * g.h * 2}, {(void**)&s.expert_sum, B * g.lh * 4},
      {(void**)&s.fix_part, (size_t)g.fix_bank * 2 * 4}, {(void**)&s.argmax_key, B * 8},
      {(void**)&s.situ_buf, situ_floats * 4},
      {(void**)&s.phase_ts, (kMaxPhases + 1) * 8}, {(void**)&s.sub_ts, (size_t)kArrivePhases * 16 * 8},
      {(void**)&s.arrive_ts, profiling ? (size_t)kArrivePhases * 1024 * 8 : 0},
      {(void**)&s.warp_ts, profiling ? (size_t)kArrivePhases * sms * kWarps * 8 : 0},
  };
  size_t off = 0;
  for (auto& it : items) {
    *it.p = (base && it.bytes) ? base + off : nullptr;
    // the exchange block's data regions are written before they are read: only its flag array must be zero
    if (it.p == (void**)&comm) pl->zero = off + (comm_inline ? flag_bytes : 0);
    off += align_up(it.bytes, 256);
  }
  pl->total = off;
  // the mirror word stands in for mapped host memory when the caller gives none (kk3_init replaces it)
  s.err_host = err_mirror;
  if (comm_inline) c.base[g.rank] = comm;
  const int HR = g.mla_mt * 16;
  size_t sm = mla_smem_bytes(HR);
  const size_t sm_row = (512 + (size_t)(g.h > g.lh ? g.h : g.lh)) * 4 + 64;
  const size_t sm_abs = ((size_t)g.B * 128 + 4 * 16 * 128) * 4;
  const size_t sm_comb = mla_combine_smem_bytes(g.B);
  const size_t sm_route = kRouteSmem;
  const size_t sm_gemv = (size_t)kWarps * kGemvSmemPerWarp;   // per-warp cp.async rings of the GEMV phases
  sm = sm_gemv > sm ? sm_gemv : sm;
  sm = sm_row > sm ? sm_row : sm;
  sm = sm_abs > sm ? sm_abs : sm;
  sm = sm_comb > sm ? sm_comb : sm;
  sm = sm_route > sm ? sm_route : sm;
  sm = (size_t)kExpSmem > sm ? (size_t)kExpSmem : sm;   // expert rings + activation row cache
  pl->smem = align_up(sm, 128);
}

extern "C" int kk3_init(const kk3_config* cfg, kk3_ctx** out) {
  if (!out) return KK3_ERR_ARG;
  *out = nullptr;
  int rc = validate(cfg);
  if (rc != KK3_OK) return rc;
  KK3_CUDA(cudaSetDevice(cfg->device));
  kk3_ctx* x = new (std::nothrow) kk3_ctx();
  if (!x) return KK3_ERR_CUDA;
  x->cfg = *cfg;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, cfg->device) != cudaSuccess) { delete x; return KK3_ERR_CUDA; }
  x->sms = prop.multiProcessorCount;
  x->grid = x->sms;
  StepPlan pl;
  plan_step(cfg, x->grid, nullptr, true, false, &pl);   // sizes
  x->scratch_bytes = pl.total;
  if (cudaMalloc(&x->scratch, pl.total) != cudaSuccess) { delete x; return KK3_ERR_CUDA; }
  if (cudaMemset(x->scratch, 0, pl.total) != cudaSuccess) { cudaFree(x->scratch); delete x; return KK3_ERR_CUDA; }
  plan_step(cfg, x->grid, (unsigned char*)x->scratch, true, false, &pl);
  x->g = pl.g;
  x->s = pl.s;
  x->nt = pl.nt;
  const Geo& g = x->g;
  Scratch& s = x->s;
  const size_t B = g.B;
  // device error word in mapped host memory, readable without synchronising
  if (cudaHostAlloc((void**)&x->err_host, 64, cudaHostAllocMapped) != cudaSuccess) {
    cudaFree(x->scratch); delete x; return KK3_ERR_CUDA;
  }
  memset(x->err_host, 0, 64);
  if (cudaHostGetDevicePointer((void**)&x->err_dev, x->err_host, 0) != cudaSuccess) {
    cudaFreeHost(x->err_host); cudaFree(x->scratch); delete x; return KK3_ERR_CUDA;
  }
  s.err_host = x->err_dev;
  if (cudaHostAlloc((void**)&x->trace_host, kTraceWords * sizeof(int), cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer((void**)&x->trace_dev, x->trace_host, 0) != cudaSuccess) {
    cudaFreeHost(x->err_host); cudaFree(x->scratch); delete x; return KK3_ERR_CUDA;
  }
  memset(x->trace_host, 0xff, kTraceWords * sizeof(int));
  s.trace_host = x->trace_dev;
  // exchange buffer: its own allocation, so that CUDA IPC can export it to the peers
  x->comm = pl.comm;
  Comm& c = x->comm;
  x->comm_bytes = pl.comm_bytes;
  if (cudaMalloc(&x->comm_local, x->comm_bytes) != cudaSuccess ||
      cudaMemset(x->comm_local, 0, x->comm_bytes) != cudaSuccess) {
    cudaFreeHost(x->err_host); cudaFree(x->scratch); delete x; return KK3_ERR_CUDA;
  }
  for (int i = 0; i < kMaxTp; ++i) c.base[i] = nullptr;
  c.base[g.rank] = (unsigned char*)x->comm_local;
  x->peers_open = g.tp == 1;
  x->smem = pl.smem;
  if (x->smem > (size_t)prop.sharedMemPerBlockOptin) {
    kk3_free(x);
    return KK3_ERR_UNSUPPORTED;
  }
  int occ = 0;
  if (prepare_kernel(x->nt, x->smem, &occ) != cudaSuccess || occ < 1) {
    kk3_free(x);
    return KK3_ERR_UNSUPPORTED;
  }
  x->args = new (std::nothrow) StepArgs();
  if (!x->args) { kk3_free(x); return KK3_ERR_CUDA; }
  // diagnostics table
  const size_t qkv_w = pl.qkv_w;
  void* bp[KK3_BUF_COUNT] = {s.prefix, s.xa, s.xm, s.attn_in, s.scores, s.latent, s.shared_act, s.x3, s.route_w,
                             s.qkv, s.mla_q, s.absorbed, s.absorbed, s.expert_sum, s.blocks, x->comm_local,
                             s.phase_ts, s.arrive_ts, s.sub_ts, s.warp_ts};
  size_t bb[KK3_BUF_COUNT] = {B * g.h * 2, B * g.h * 2, B * g.h * 2, B * (size_t)g.hr * g.vd * 2, B * g.E * 4,
                              B * g.lh * 2, B * (size_t)g.sinter * 2, B * g.lh * 2, B * g.K * 4, B * qkv_w * 2,
                              B * (size_t)g.hr * (g.nr + g.rd) * 2, B * (size_t)g.hr * g.kr * 2,
                              B * (size_t)g.hr * g.kr * 2, B * g.lh * 4, (size_t)g.nblk * B * g.h * 2, x->comm_bytes,
                              (size_t)(kMaxPhases + 1) * 8, (size_t)kArrivePhases * 1024 * 8,
                              (size_t)kArrivePhases * 16 * 8, (size_t)kArrivePhases * x->grid * kWarps * 8};
  for (int i = 0; i < KK3_BUF_COUNT; ++i) { x->buf_ptr[i] = bp[i]; x->buf_bytes[i] = bb[i]; }
  *out = x;
  return KK3_OK;
}

extern "C" int kk3_ipc_handle(kk3_ctx* x, void* handle64) {
  if (!x || !handle64) return KK3_ERR_ARG;
  KK3_CUDA(cudaSetDevice(x->cfg.device));
  cudaIpcMemHandle_t h;
  KK3_CUDA(cudaIpcGetMemHandle(&h, x->comm_local));
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(handle64, &h, 64);
  return KK3_OK;
}

extern "C" int kk3_open_peers(kk3_ctx* x, const void* handles) {
  if (!x || !handles) return KK3_ERR_ARG;
  KK3_CUDA(cudaSetDevice(x->cfg.device));
  for (int r = 0; r < x->g.tp; ++r) {
    if (r == x->g.rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, (const char*)handles + 64 * r, 64);
    void* p = nullptr;
    KK3_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    x->peer_open[r] = p;
    x->comm.base[r] = (unsigned char*)p;
  }
  x->peers_open = 1;
  return KK3_OK;
}

// Single-process testing aid: use an existing device allocation as rank r's exchange buffer.
extern "C" int kk3_debug_set_peer(kk3_ctx* x, int r, void* device_ptr) {
  if (!x || r < 0 || r >= x->g.tp || r == x->g.rank || !device_ptr) return KK3_ERR_ARG;
  x->comm.base[r] = (unsigned char*)device_ptr;
  int all = 1;
  for (int i = 0; i < x->g.tp; ++i) all &= x->comm.base[i] != nullptr;
  x->peers_open = all;
  return KK3_OK;
}

extern "C" size_t kk3_exchange_bytes(kk3_ctx* x) { return x ? x->comm_bytes : 0; }

extern "C" int kk3_exchange_layout(kk3_ctx* x, long long* offsets) {
  if (!x || !offsets) return KK3_ERR_ARG;
  const Comm& c = x->comm;
  const long long v[8] = {c.flag_off, c.data_off[0], c.data_off[1], c.region_bytes,
                          c.att_off, c.exp_off, c.shd_off, c.key_off};
  for (int i = 0; i < 8; ++i) offsets[i] = v[i];
  return KK3_OK;
}

extern "C" int kk3_set_comm_mode(kk3_ctx* x, int mode) {
  if (!x || (mode != KK3_COMM_PEER && mode != KK3_COMM_HOST && mode != KK3_COMM_PUSH)) return KK3_ERR_ARG;
  x->comm_mode = mode == KK3_COMM_HOST ? kCommHost : (mode == KK3_COMM_PUSH ? kCommPush : kCommPeer);
  return KK3_OK;
}

extern "C" int kk3_set_gemv_engine(kk3_ctx* x, int engine) {
  if (!x || (engine != KK3_GEMV_AUTO && engine != KK3_GEMV_MMA)) return KK3_ERR_ARG;
  x->gemv_engine = engine == KK3_GEMV_MMA ? kGemvMma : kGemvAuto;
  return KK3_OK;
}

// Every tensor except the token ids and reset flags is read with 16-byte vector or cp.async loads, so a
// misaligned pointer would fault on the device: reject it here instead.
static bool table_aligned(const void* const* table, int n) {
  for (int i = 0; i < n; ++i) {
    if (i == KK3_TOKEN || i == KK3_RESET) continue;
    if (reinterpret_cast<uintptr_t>(table[i]) & 15u) return false;
  }
  return true;
}

// Slots the geometry reads or writes (the runtime's table layout): the global inputs, the outputs (the MLA
// cache rows only with MLA layers, the KDA states only with KDA layers), and per layer its attention block
// (MLA or KDA) and its FFN block (dense or MoE). Every one of them must be non-NULL; the rest may be NULL.
static bool slot_required(const Geo& g, int i) {
  if (i < KK3_GLOBAL_SLOTS) {
    if (i == KK3_OUT_KV_WRITE || i == KK3_OUT_PE_WRITE) return g.nmla > 0;
    if (i == KK3_OUT_RECURRENT_STATE || i == KK3_OUT_CONV_STATE) return g.nkda > 0;
    return i <= KK3_OUT_CACHE_LENGTH;
  }
  const int l = (i - KK3_GLOBAL_SLOTS) / KK3_LAYER_SLOTS, s = (i - KK3_GLOBAL_SLOTS) % KK3_LAYER_SLOTS;
  const bool mla = ((l + 1) % 4 == 0) || l == g.L - 1;
  if (s < KK3_DENSE_GATE) return s <= (mla ? (int)KK3_MLA_PE_CACHE : (int)KK3_KDA_RECURRENT_STATE);
  return s <= (l < g.first_dense ? (int)KK3_DENSE_DOWN : (int)KK3_MOE_SHARED_DOWN);
}

static bool table_complete(const void* const* table, int n, const Geo& g) {
  for (int i = 0; i < n; ++i)
    if (table[i] == nullptr && slot_required(g, i)) return false;
  return true;
}

extern "C" int kk3_check_table(const kk3_config* cfg, const void* const* table, int table_size) {
  const int rc = validate(cfg);
  if (rc != KK3_OK) return rc;
  if (!table || table_size != KK3_GLOBAL_SLOTS + cfg->layers * KK3_LAYER_SLOTS || table_size > kMaxPtrs ||
      !table_aligned(table, table_size))
    return KK3_ERR_ARG;
  Geo g{};
  g.L = cfg->layers;
  g.first_dense = cfg->first_dense;
  for (int l = 0; l < g.L; ++l) {
    if (((l + 1) % 4 == 0) || l == g.L - 1) ++g.nmla; else ++g.nkda;
  }
  return table_complete(table, table_size, g) ? KK3_OK : KK3_ERR_ARG;
}

static int launch(kk3_ctx* x, const void* const* table, int n, void* stream, int stop_phase, int start_phase,
                  const long long* lengths = nullptr) {
  if (!x || !table) return KK3_ERR_ARG;
  if (x->failed) return KK3_ERR_FAILED;
  if (!x->peers_open) return KK3_ERR_PEERS;
  const int need = KK3_GLOBAL_SLOTS + x->g.L * KK3_LAYER_SLOTS;
  if (n != need || n > kMaxPtrs || !table_aligned(table, n) || !table_complete(table, n, x->g)) return KK3_ERR_ARG;
  if (*x->err_host != 0) {
    x->failed = 1;
    return KK3_ERR_FAILED;
  }
  StepArgs* a = x->args;
  a->g = x->g;
  a->s = x->s;
  a->comm = x->comm;
  a->epoch = ++x->epoch;
  a->stop_phase = stop_phase;
  a->start_phase = start_phase < 0 ? 0 : start_phase;
  a->trace = x->trace;
  a->comm_mode = x->comm_mode;
  a->gemv_engine = x->gemv_engine;
  a->lengths = lengths;
  a->nptr = n;
  memcpy(a->ptr, table, sizeof(void*) * n);
  cudaError_t e = launch_kernel(x->nt, a, x->grid, x->smem, (cudaStream_t)stream);
  return cuda_fail(e, "cudaLaunchCooperativeKernel(kk3_step_kernel)");
}

extern "C" int kk3_step(kk3_ctx* x, const void* const* table, int n, void* stream) {
  return launch(x, table, n, stream, -1, 0);
}

extern "C" int kk3_step_append(kk3_ctx* x, const void* const* table, int n, const int64_t* lengths, void* stream) {
  if (!x || !lengths || (reinterpret_cast<uintptr_t>(lengths) & 7u)) return KK3_ERR_ARG;
  return launch(x, table, n, stream, -1, 0, reinterpret_cast<const long long*>(lengths));
}

extern "C" int kk3_debug_step(kk3_ctx* x, const void* const* table, int n, void* stream, int stop_phase) {
  return launch(x, table, n, stream, stop_phase < 0 ? -1 : stop_phase, 0);
}

extern "C" int kk3_debug_phases(kk3_ctx* x, const void* const* table, int n, void* stream, int start_phase,
                                int stop_phase) {
  return launch(x, table, n, stream, stop_phase < 0 ? -1 : stop_phase, start_phase);
}

extern "C" int kk3_status(kk3_ctx* x) {
  if (!x) return KK3_ERR_ARG;
  const int e = *(volatile int*)x->err_host;
  if (e == kErrTimeout) { x->failed = 1; return KK3_ERR_TIMEOUT; }
  if (e != 0) { x->failed = 1; return KK3_ERR_DEVICE; }
  return KK3_OK;
}

extern "C" int kk3_phase_count(kk3_ctx* x) {
  if (!x) return KK3_ERR_ARG;
  int v = 0;
  if (cudaMemcpy(&v, x->s.phase_count, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return KK3_ERR_CUDA;
  return v;
}

extern "C" int kk3_debug_buffer(kk3_ctx* x, int id, void** ptr, size_t* bytes) {
  if (!x || id < 0 || id >= KK3_BUF_COUNT || !ptr || !bytes) return KK3_ERR_ARG;
  *ptr = x->buf_ptr[id];
  *bytes = x->buf_bytes[id];
  return KK3_OK;
}

extern "C" int kk3_debug_copy(kk3_ctx* x, int id, void* dst, size_t bytes) {
  if (!x || id < 0 || id >= KK3_BUF_COUNT || !dst || bytes > x->buf_bytes[id]) return KK3_ERR_ARG;
  KK3_CUDA(cudaSetDevice(x->cfg.device));
  KK3_CUDA(cudaMemcpy(dst, x->buf_ptr[id], bytes, cudaMemcpyDeviceToDevice));
  return KK3_OK;
}

extern "C" int kk3_debug_trace(kk3_ctx* x, int enable, int* out, int n) {
  if (!x) return KK3_ERR_ARG;
  if (enable >= 0) x->trace = enable;
  if (out) {
    const int m = n < kTraceWords ? n : kTraceWords;
    for (int i = 0; i < m; ++i) out[i] = ((volatile int*)x->trace_host)[i];
  }
  return KK3_OK;
}

extern "C" void kk3_free(kk3_ctx* x) {
  if (!x) return;
  cudaSetDevice(x->cfg.device);
  for (int r = 0; r < kMaxTp; ++r)
    if (x->peer_open[r]) cudaIpcCloseMemHandle(x->peer_open[r]);
  if (x->comm_local) cudaFree(x->comm_local);
  if (x->scratch) cudaFree(x->scratch);
  if (x->err_host) cudaFreeHost(x->err_host);
  if (x->trace_host) cudaFreeHost(x->trace_host);
  delete x->args;
  delete x;
}

extern "C" int kk3_launch_config(kk3_ctx* x, int* grid, int* threads, size_t* smem) {
  if (!x) return KK3_ERR_ARG;
  if (grid) *grid = x->grid;
  if (threads) *threads = kThreads;
  if (smem) *smem = x->smem;
  return KK3_OK;
}

// ---------------------------------------------------------------------------------------------------------
// kk3_step_noalloc: the decode step with its scratch in one file-scope device array instead of memory that
// kk3_init allocates. No counterpart in the reference.
//
// Who needs it: callers that cannot allocate device memory when they run a step. A serving engine hands
// nearly all of HBM to its own caches and memory pool before the first request, so a later cudaMalloc of
// tens of MB fails or fragments that pool; and a latency-bound loop must not call cudaMalloc or cudaFree,
// because both synchronise the whole device and stall every other stream on it.
//
// What it does not do: allocate. No cudaMalloc, cudaHostAlloc, cudaFree or allocating library routine (torch
// included) runs on this path; only cudaGetSymbolAddress, kernel attribute and occupancy queries (first call
// per device), cudaMemsetAsync of the scratch and the cooperative launch.
//
// Limits: tp == 1 only, because CUDA IPC cannot export a static device symbol, so tensor-parallel peers
// would have no exchange buffer to map. The scratch the geometry needs must fit kNoAllocScratchBytes
// (32 MiB), which holds one TP8 rank's shapes at batch <= 8 and every small test geometry; larger
// geometries get KK3_ERR_TOO_LARGE and should use kk3_init + kk3_step.
//
// Concurrency: there is one scratch array per device. Two calls whose steps overlap on one device (other
// streams, other host threads) race on it and corrupt each other; serialise them.
namespace kk3 {

cudaError_t raise_smem_nt1(size_t smem);
cudaError_t raise_smem_nt2(size_t smem);
cudaError_t raise_smem_nt4(size_t smem);
cudaError_t raise_smem_nt8(size_t smem);

constexpr size_t kNoAllocScratchBytes = 32ull << 20;
static __device__ __align__(256) unsigned char kk3_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kNoAllocMaxDevices = 64;
struct NoAllocDevice {
  int ready = 0;
  unsigned char* base = nullptr;   // device address of kk3_noalloc_scratch on this device
  int sms = 0;
  size_t smem_optin = 0;
  unsigned epoch = 0;
  kk3_config last = {};            // geometry of the previous call on this device
  int has_last = 0;
};
static NoAllocDevice noalloc_dev[kNoAllocMaxDevices];
static std::mutex noalloc_mu;

// First call on a device, with that device current: find the scratch array's device address and the SM
// count. The first call therefore does CUDA set-up work; make it before any stream capture that contains
// this entry point and before latency-sensitive use.
static int noalloc_setup(int device, NoAllocDevice* d) {
  if (d->ready) return KK3_OK;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, kk3_noalloc_scratch);
  if (e != cudaSuccess || !p) return cuda_fail(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                                               "cudaGetSymbolAddress(kk3_noalloc_scratch)");
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  d->base = (unsigned char*)p;
  d->sms = prop.multiProcessorCount;
  d->smem_optin = prop.sharedMemPerBlockOptin;
  d->ready = 1;
  return KK3_OK;
}

}  // namespace kk3

extern "C" int kk3_step_noalloc(const kk3_config* cfg, const void* const* table, int table_size, void* stream,
                                int* error_word) {
  int rc = validate(cfg);
  if (rc != KK3_OK) return rc;
  if (cfg->tp != 1 || cfg->rank != 0) return KK3_ERR_UNSUPPORTED;
  if (!table || table_size != KK3_GLOBAL_SLOTS + cfg->layers * KK3_LAYER_SLOTS || table_size > kMaxPtrs ||
      !table_aligned(table, table_size))
    return KK3_ERR_ARG;
  if (cfg->device < 0 || cfg->device >= kNoAllocMaxDevices) return KK3_ERR_ARG;
  std::lock_guard<std::mutex> lock(noalloc_mu);   // host-side state only; see the concurrency note above
  int prev = -1;
  KK3_CUDA(cudaGetDevice(&prev));
  if (prev != cfg->device) KK3_CUDA(cudaSetDevice(cfg->device));
  struct Restore {
    int dev;
    bool on;
    ~Restore() { if (on) cudaSetDevice(dev); }
  } restore{prev, prev != cfg->device};
  NoAllocDevice* d = &noalloc_dev[cfg->device];
  rc = noalloc_setup(cfg->device, d);
  if (rc != KK3_OK) return rc;
  // the argument block is ~25 KB (one pointer per table slot); it lives on this host stack until the launch
  // has copied it
  StepArgs a;
  StepPlan pl;
  plan_step(cfg, d->sms, d->base, false, true, &pl);   // the same planner as kk3_init
  const size_t total = pl.total, zero = pl.zero, smem = pl.smem;
  const int nt = pl.nt;
  a.g = pl.g;
  a.s = pl.s;
  a.comm = pl.comm;
  if (total > kNoAllocScratchBytes) return KK3_ERR_TOO_LARGE;
  if (smem > d->smem_optin) return KK3_ERR_UNSUPPORTED;
  if (!table_complete(table, table_size, a.g)) return KK3_ERR_ARG;   // before anything is cleared or launched
  // The kernel's dynamic shared memory limit is per-function state shared with kk3_init; both raise it when
  // below the launch's need and never lower it, so every live context keeps working.
  {
    cudaError_t e = nt == 1 ? raise_smem_nt1(smem) : nt == 2 ? raise_smem_nt2(smem)
                  : nt == 4 ? raise_smem_nt4(smem) : raise_smem_nt8(smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(kk3_step_kernel)");
  }
  cudaStream_t st = (cudaStream_t)stream;
  // Zero state. The barrier word, phase count, error words, stream-K tile counters and exchange flags must
  // be zero when a step begins; a completed step leaves them so, a failed one may not, so they are cleared
  // before every launch. When the geometry differs from the previous call's, the whole planned scratch is
  // cleared once, so nothing a previous geometry left behind is seen.
  const bool same = d->has_last && memcmp(&d->last, cfg, sizeof(kk3_config)) == 0;
  KK3_CUDA(cudaMemsetAsync(d->base, 0, same ? zero : total, st));
  d->last = *cfg;
  d->has_last = 1;
  if (error_word) a.s.err_host = error_word;
  a.epoch = ++d->epoch;
  a.stop_phase = -1;
  a.start_phase = 0;
  a.trace = 0;
  a.comm_mode = kCommPeer;
  a.gemv_engine = kGemvAuto;
  a.lengths = nullptr;
  a.nptr = table_size;
  memcpy(a.ptr, table, sizeof(void*) * table_size);
  cudaError_t e = launch_kernel(nt, &a, d->sms, smem, st);
  return cuda_fail(e, "cudaLaunchCooperativeKernel(kk3_step_kernel)");
}
