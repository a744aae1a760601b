// kk3_common.cuh - shared device types and PTX helpers for the sm_100a Kimi K3 decode-step kernel.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/kk3.h"

#define KK3_DEV __device__ __forceinline__
// Phase engines are real functions: one shared copy stays hot in the instruction cache across phases and
// layers (inlining a copy per call site made every phase run cold code).
#define KK3_FN static __device__ __noinline__

namespace kk3 {

typedef __nv_bfloat16 bf16;

constexpr int kThreads = 512;          // one CTA per SM, 16 warps
constexpr int kWarps = kThreads / 32;
constexpr int kMaxBatch = 64;
constexpr int kMaxTp = 8;
constexpr int kMaxTopk = 32;
constexpr int kMaxExperts = 1024;
constexpr int kMaxPtrs = KK3_GLOBAL_SLOTS + 96 * KK3_LAYER_SLOTS;   // 3104 slots: up to 96 layers
constexpr int kMlaPos = 32;            // cache positions per attention sub-tile
constexpr int kMaxPhases = 2048;       // phase timestamp capacity (a 96-layer step has ~1500 phases)
constexpr int kArrivePhases = 256;     // phases with per-CTA barrier arrival stamps
constexpr int kTraceWords = 2 * 1024 + 4096;   // mapped trace: phase and progress per CTA, marker per warp

// exchange transport (StepArgs::comm_mode)
constexpr int kCommPeer = 0;   // in-kernel one-shot NVLink peer stores + per-row release flags (the product)
constexpr int kCommHost = 1;   // comparison baseline: the host runs NCCL collectives between phase-range launches
constexpr int kCommPush = 2;   // in-kernel, with the GEMV partials stored locally and pushed to the peers in coalesced
                               // per-CTA chunks at the start of the phase that reads them (release flag per chunk)

// device error word values (also the host-visible status)
constexpr int kErrTimeout = 1;
constexpr int kErrDevice = 2;

// ---------------------------------------------------------------------------------------------
// Geometry and scratch layout, copied into the kernel parameters.

struct Geo {
  int L, B, h, lh, inter, dinter, sinter, hr, d, qr, kr, nr, rd, vd, V, E, K, ctx, conv, bs, first_dense;
  int tp, rank;
  int qdim;          // hr * d
  int nmla, nkda;    // layer counts
  int nblk;          // block-vector capacity
  long long timeout_ns;
  int mla_chunks;    // split-K chunks per batch row of the MLA attention
  int mla_chunk_len; // positions per chunk (multiple of kMlaPos)
  long long fix_bank; // floats per stream-K partial bank (two banks: two GEMV passes may share a phase)
  int cnt_bank;       // counters per stream-K counter bank
  int mla_mt;         // 16-row head tiles per head group of the MLA attention (<= 4)
  int mla_groups;     // head groups: ceil(ceil(hr / 16) / mla_mt)
  int bp;             // batch padded to the step's n-tile width (8 * NT): the bf16 exchange regions' batch stride
};

// scratch buffers (device pointers owned by the context)
struct Scratch {
  bf16* prefix;       // [B, h]
  bf16* blocks;       // [nblk, B, h]
  bf16* xa;           // [B, h]   normalised attention input
  bf16* xm;           // [B, h]   normalised MLP input
  bf16* qkv;          // [B, 3*qdim] KDA q,k,v projections (or MLA qa [B,qr] + ka [B,576])
  bf16* og;           // [B, qdim] output-gate projection
  bf16* fa;           // [B, d]
  bf16* beta;         // [B, hr]
  bf16* attn_in;      // [B, hr*vd] input of the o projection
  bf16* mla_qan;      // [B, qr]
  bf16* mla_q;        // [B, hr*(nr+rd)]
  bf16* absorbed;     // [B, hr, kr]
  float* mla_part;    // [B, chunks, hr, kr+2]
  bf16* dense_act;    // [B, dinter]
  float* scores;      // [B, E] sigmoid router scores (FP32)
  bf16* latent;       // [B, lh]
  __half* latent_p;   // [B, lh] FP16 copy of the latent: the activation operand of the MXFP4 experts
  bf16* shared_act;   // [B, sinter]
  int* route_ids;     // [B, K] sorted expert ids of the current layer
  float* route_w;     // [B, K] renormalised weights (same order)
  int* pair_row;      // [B*K] pair -> batch row, grouped by expert
  int* pair_slot;     // [B*K] pair -> slot j
  int* chunk_info;    // [1 + B*K*3]: count, then (expert, first pair, pairs) per expert chunk of <= 8 pairs
  __half* act_p;      // [B*K, inter] FP16 expert activations (operand of the down projection)
  bf16* out_slot;     // [B, K, lh] per-slot expert outputs
  bf16* x3;           // [B, lh] latent_norm(expert_sum)
  bf16* shared_red;   // [B, h] reduced shared-expert output
  float* expert_sum;  // [B, lh] FP32 (diagnostics copy of the local sum)
  float* fix_part;    // [2 * warps_total, 16 * 64 * 2] stream-K partial tiles
  int* fix_cnt;       // [max tiles] stream-K arrival counters
  unsigned long long* argmax_key; // [B]
  float* situ_buf;    // [2 halves][tiles][32 lanes][4 * NT] bf16-rounded gate / up tiles of a situ pair
  int* situ_cnt;      // [tiles] halves of a situ pair published (the second resets it)
  unsigned* bar;      // grid barrier word (see grid_sync)
  int* err;           // device error word, polled by every wait (device memory: cheap to poll)
  int* err_host;      // host-visible copy in mapped host memory, written only when an error is raised
  int* phase_count;   // number of grid phases of the last complete step
  unsigned long long* phase_ts;  // [kMaxPhases + 1] globaltimer at kernel start and at the end of each phase
  unsigned long long* arrive_ts; // [kArrivePhases][grid] barrier arrival time of every CTA (profiling)
  unsigned long long* warp_ts;   // [kArrivePhases][grid][kWarps] time each engine warp finished (profiling)
  unsigned long long* sub_ts;    // [kArrivePhases][16] sub-phase stamps of one CTA / warp (profiling)
  int* trace_host;    // mapped host memory [2][1024]: per-CTA phase and progress, readable after a fault
};

// One-shot exchange buffers, symmetric across ranks (this rank's and peers' mapped copies).
struct Comm {
  unsigned char* base[kMaxTp];   // per rank, this rank's view of rank r's exchange buffer
  long long flag_off;            // byte offset of the flag array [B][tp] (u32)
  long long push_flag_off;       // byte offset of the chunk-push flag array [tp][grid] (u32), push transport
  long long data_off[2];         // byte offset of the two parity data regions
  long long region_bytes;        // bytes per parity region
  // sub-regions inside a parity region, byte offsets (each [tp][B][width])
  long long att_off, exp_off, shd_off, key_off;
};

constexpr int kGemvAuto = 0, kGemvMma = 1;

struct StepArgs {
  Geo g;
  Scratch s;
  Comm comm;
  unsigned epoch;       // step counter (1, 2, ...), orders the peer flags
  int stop_phase;       // debug: return after this many grid phases (-1: run everything)
  int start_phase;      // debug: skip the work (and barriers) of phases before this one (0: run everything)
  int trace;            // debug: publish per-CTA progress to mapped host memory (fault localisation)
  int comm_mode;        // kCommPeer: one-shot peer stores and flags inside the kernel; kCommHost: each rank
                        // writes only its own slot and the host reduces the slots between launches (NCCL)
  const long long* lengths;   // append mode (kk3_step_append): cached positions of each row, [B]; null otherwise
  int gemv_engine;      // kGemvAuto: tcgen05 projections for batches above 16, mma.sync below; kGemvMma: mma.sync
                        // for every batch (the comparison engine)
  int nptr;
  const void* ptr[kMaxPtrs];
};

// ---------------------------------------------------------------------------------------------
// small helpers

KK3_DEV unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

KK3_DEV unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

KK3_DEV unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

KK3_DEV void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

KK3_DEV int ld_volatile_int(const int* p) { return *(volatile const int*)p; }

// streaming 16-byte weight load: read-only path, no L1 allocation
KK3_DEV uint4 ldg_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
KK3_DEV unsigned ldg_nc32(const void* p) {
  unsigned v;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
KK3_DEV unsigned ldg_nc16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
KK3_DEV unsigned ldg_nc8(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u8 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}
// activation load: coherent global load (data written earlier in this kernel, ordered by a grid barrier)
KK3_DEV uint4 ld_act16(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
// L2-only load for data another CTA may have written after this SM cached the line
KK3_DEV float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

KK3_DEV float bf2f(bf16 v) { return __bfloat162float(v); }
KK3_DEV bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
KK3_DEV float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

KK3_DEV float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// E8M0 scale byte -> 2^(s-127) in FP32; 255 is NaN (megabench/tasks/quantization.py:49-50)
KK3_DEV float e8m0_to_f32(unsigned s) {
  float v = __uint_as_float(s << 23);
  v = (s == 0u) ? 5.877471754111438e-39f : v;
  v = (s == 255u) ? __uint_as_float(0x7fc00000u) : v;
  return v;
}

// D = A*B + C, m16n8k16, BF16 inputs, FP32 accumulate
KK3_DEV void mma_bf16(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
KK3_DEV void mma_f16(float (&d)[4], unsigned a0, unsigned a1, unsigned a2, unsigned a3, unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

KK3_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
KK3_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// CTA-wide sum of one float (all threads get the result). `red` needs kWarps floats of shared memory.
KK3_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kWarps ? red[lane] : 0.0f;
  return warp_sum(t);
}

// profiling stamp `k` (< 16) of the current phase, written by the calling thread
KK3_DEV void sub_stamp(const StepArgs& a, int phase, int k, unsigned long long v = 0) {
  if (phase >= 0 && phase < kArrivePhases) a.s.sub_ts[phase * 16 + k] = v ? v : globaltimer();
}

// fault localisation: thread 0 of each CTA publishes (slot 0) its phase and (slot 1) a progress code
KK3_DEV void trace_progress(const StepArgs& a, int which, int value) {
  if (a.trace && threadIdx.x == 0) {
    reinterpret_cast<volatile int*>(a.s.trace_host)[which * 1024 + blockIdx.x] = value;
    __threadfence_system();
  }
}
// the grid phase this CTA is in, for the engines' profiling stamps (set at kernel start and by grid_sync)
static __shared__ int kk3_cur_phase;

// lane 0 of an engine warp records when the warp finished its share of the phase (profiling only)
KK3_DEV void warp_end_stamp(const StepArgs& a) {
  if (a.s.warp_ts && (threadIdx.x & 31) == 0) {
    const int ph = kk3_cur_phase;
    if (ph >= 0 && ph < kArrivePhases)
      a.s.warp_ts[((size_t)ph * gridDim.x + blockIdx.x) * kWarps + (threadIdx.x >> 5)] = globaltimer();
  }
}

// per-warp marker (lane 0), for locating a fault inside an engine; only when tracing is enabled
KK3_DEV void trace_warp(const StepArgs& a, int value) {
  if (a.trace && (threadIdx.x & 31) == 0) {
    const int w = blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (w < 4096) {
      reinterpret_cast<volatile int*>(a.s.trace_host)[2 * 1024 + w] = value;
      __threadfence_system();
    }
  }
}

// pointer-table access
template <typename T>
KK3_DEV const T* gptr(const StepArgs& a, int slot) { return reinterpret_cast<const T*>(a.ptr[slot]); }
template <typename T>
KK3_DEV const T* lptr(const StepArgs& a, int layer, int slot) {
  return reinterpret_cast<const T*>(a.ptr[KK3_GLOBAL_SLOTS + layer * KK3_LAYER_SLOTS + slot]);
}
template <typename T>
KK3_DEV T* gout(const StepArgs& a, int slot) { return reinterpret_cast<T*>(const_cast<void*>(a.ptr[slot])); }

// Cached MLA positions row b attends: 0 after a reset; in append mode its length from `lengths` (clamped to the
// cache capacity; kk3_step_append requires lengths[b] < context); else the whole context (kimi.py:274-280).
KK3_DEV int mla_row_len(const StepArgs& a, int b) {
  if (reinterpret_cast<const bool*>(a.ptr[KK3_RESET])[b]) return 0;
  if (a.lengths == nullptr) return a.g.ctx;
  const long long n = a.lengths[b];
  return n < 0 ? 0 : (n > a.g.ctx ? a.g.ctx : (int)n);
}
// split-K chunks of row b: its attended sequence (cached positions + the new token) in chunks of mla_chunk_len
KK3_DEV int mla_row_chunks(const StepArgs& a, int b) {
  return (mla_row_len(a, b) + 1 + a.g.mla_chunk_len - 1) / a.g.mla_chunk_len;
}

KK3_DEV void set_error(const StepArgs& a, int code) {
  if (atomicCAS(a.s.err, 0, code) == 0) {
    *reinterpret_cast<volatile int*>(a.s.err_host) = code;
    __threadfence_system();
  }
}
KK3_DEV bool failed(const StepArgs& a) { return ld_volatile_int(a.s.err) != 0; }

// Bounded grid-wide barrier on one 32-bit word. Every CTA adds 1, except CTA 0 which adds 2^31 - (G - 1), so
// the word advances by exactly 2^31 per barrier and its top bit flips once all G CTAs have arrived: one
// atomic per CTA, no reset. The arrival is a release RMW (the CTA's writes, ordered before it by the CTA
// barrier, become visible with it) and the waiters poll with acquire loads, so no separate fences sit on the
// critical path. The error word is checked every 64 polls and the wait gives up after timeout_ns. Returns
// false on timeout or a reported error; the kernel unwinds. When `arrive_ts` is set, each CTA stamps its
// arrival time (phase profiling).
KK3_DEV unsigned atom_add_release_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.release.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

KK3_DEV int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

KK3_FN bool grid_sync(const StepArgs& a, int phase = -1) {
  __shared__ int ok_flag;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned* word = a.s.bar;
    int ok = 1;
    if (a.s.arrive_ts && phase >= 0 && phase < kArrivePhases)
      a.s.arrive_ts[(size_t)phase * gridDim.x + blockIdx.x] = globaltimer();
    const unsigned add = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1) : 1u;
    const unsigned old = atom_add_release_gpu(word, add);
    unsigned long long t0 = 0;
    for (unsigned spin = 0;; ++spin) {
      if (((old ^ ld_acquire_gpu(word)) & 0x80000000u) != 0) break;
      // after ~20 us of polling (long tails), back off so the waiters do not keep the word's L2 slice busy
      if (spin >= 32) __nanosleep(64);
      if ((spin & 63) == 63) {
        const unsigned long long t = globaltimer();
        if (t0 == 0) t0 = t;
        if (failed(a) || t - t0 > (unsigned long long)a.g.timeout_ns) {
          set_error(a, kErrTimeout);
          ok = 0;
          break;
        }
      }
    }
    ok_flag = ok;
    kk3_cur_phase = phase + 1;
  }
  __syncthreads();
  return ok_flag != 0;
}

// Wait (thread-level) until *flag >= want (system scope). Returns false on timeout / error.
KK3_DEV bool wait_flag_sys(const StepArgs& a, const unsigned* flag, unsigned want) {
  const unsigned long long t0 = globaltimer();
  while ((int)(ld_acquire_sys(flag) - want) < 0) {
    if (failed(a) || globaltimer() - t0 > (unsigned long long)a.g.timeout_ns) {
      set_error(a, kErrTimeout);
      return false;
    }
    __nanosleep(32);
  }
  return true;
}

}  // namespace kk3
