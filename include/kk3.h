/*
 * kk3.h - C ABI of the B200 (sm_100a) Kimi K3 decode step, one tensor-parallel rank per context.
 *
 * This is the drop-in boundary beneath MegaBench's submission interface
 * (garv901/kimi-k3-goalbox megabench/harness/runner.py:53-69: `build(case) -> run(inputs) -> outputs`).
 * The Python host (`kimi_k3_goalbox_b200/submission.py`) calls these entry points through ctypes; no
 * torch types cross this boundary, only plain device pointers, sizes and a CUDA stream handle.
 *
 * The step computed is the reference oracle `megabench/tasks/kimi.py:230-340` (`reference(case, values)`)
 * for this rank's shard; inputs and outputs use exactly the reference's layouts (`kimi.py:72-122`,
 * `:164-182`, `:332-340`).
 */
#ifndef KK3_H
#define KK3_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Geometry of one rank. Field meanings follow the reference's case params (megabench/cases.py:48-55)
 * after tensor-parallel division (megabench/tasks/kimi.py:72-122). */
typedef struct kk3_config {
    int32_t layers;              /* params['layers'] */
    int32_t batch;               /* params['batch'] (1..64) */
    int32_t hidden;              /* params['hidden'] */
    int32_t latent_hidden;       /* params['latent_hidden'] */
    int32_t inter_shard;         /* params['intermediate'] / tp: routed-expert rows on this rank */
    int32_t dense_inter_shard;   /* params['dense_intermediate'] / tp */
    int32_t shared_inter_shard;  /* params['intermediate'] * params['shared_experts'] / tp */
    int32_t heads;               /* params['q_heads'] / tp */
    int32_t head_dim;            /* params['head_dim'] (128) */
    int32_t q_lora_rank;         /* params['q_lora_rank'] */
    int32_t kv_lora_rank;        /* params['kv_lora_rank'] (512) */
    int32_t qk_nope_dim;         /* params['qk_nope_dim'] (128) */
    int32_t qk_rope_dim;         /* params['qk_rope_dim'] (64) */
    int32_t v_head_dim;          /* params['v_head_dim'] (128) */
    int32_t vocab_shard;         /* params['vocab'] / tp */
    int32_t experts;             /* params['experts'] (<= 1024) */
    int32_t topk;                /* params['topk'] (<= 32) */
    int32_t context;             /* params['context'] (cached MLA positions) */
    int32_t conv_kernel;         /* params['conv_kernel'] (4) */
    int32_t attn_res_block_size; /* params['attn_res_block_size'] */
    int32_t first_dense;         /* params['first_dense'] */
    int32_t tp;                  /* tensor-parallel degree (1..8) */
    int32_t rank;                /* this rank's tp_rank */
    int32_t device;              /* CUDA device ordinal this context runs on */
    int64_t timeout_ns;          /* bound on every in-kernel wait (grid barrier, peer flag); 0 = default */
} kk3_config;

typedef struct kk3_ctx kk3_ctx;

/* Return codes: 0 or negative. */
#define KK3_OK               0
#define KK3_ERR_ARG         (-1)  /* bad argument or pointer table */
#define KK3_ERR_UNSUPPORTED (-2)  /* geometry outside what the kernels implement */
#define KK3_ERR_CUDA        (-3)  /* a CUDA runtime call failed */
#define KK3_ERR_TIMEOUT     (-4)  /* an in-kernel wait ran past timeout_ns (a peer or CTA never arrived) */
#define KK3_ERR_DEVICE      (-5)  /* an in-kernel consistency check failed */
#define KK3_ERR_PEERS       (-6)  /* tp > 1 and the peer buffers are not open yet */
#define KK3_ERR_FAILED      (-7)  /* an earlier step failed; the context must be freed and rebuilt */
#define KK3_ERR_TOO_LARGE   (-8)  /* kk3_step_noalloc: the geometry's scratch exceeds its static buffer */

/* Pointer table. kk3_step takes one device pointer per slot, in this order:
 *   slots [0, KK3_GLOBAL_SLOTS): the global inputs and the outputs (enum below);
 *   then KK3_LAYER_SLOTS slots per layer l at KK3_GLOBAL_SLOTS + l*KK3_LAYER_SLOTS + slot.
 * Every tensor must be contiguous, on the context's device, with the reference's shape and dtype
 * (kimi.py:72-122 weights, :164-182 state, :332-340 outputs). Slots the geometry does not use may be NULL
 * (per layer: the other attention kind's and the other FFN kind's slots; the MLA cache outputs without MLA
 * layers, the KDA state outputs without KDA layers); every used slot must be non-NULL. Every pointer except
 * KK3_TOKEN and KK3_RESET must be 16-byte aligned (read with 16-byte vector loads). The step entry points
 * return KK3_ERR_ARG for a NULL used slot or a misaligned pointer, before launching anything. */
enum kk3_global_slot {
    KK3_TOKEN = 0, KK3_RESET, KK3_EMBED, KK3_LM_HEAD, KK3_FNORM, KK3_OUTPUT_RES_NORM, KK3_OUTPUT_RES_PROJ,
    KK3_LN1, KK3_LN2, KK3_ATTENTION_RES_NORM, KK3_MLP_RES_NORM, KK3_ATTENTION_RES_PROJ, KK3_MLP_RES_PROJ,
    /* outputs */
    KK3_OUT_LOGITS, KK3_OUT_NEXT_TOKEN, KK3_OUT_KV_WRITE, KK3_OUT_PE_WRITE, KK3_OUT_RECURRENT_STATE,
    KK3_OUT_CONV_STATE, KK3_OUT_EXPERT_IDS, KK3_OUT_CACHE_LENGTH,
    KK3_GLOBAL_SLOTS = 32
};
enum kk3_layer_slot {
    /* KDA attention (kimi.py:99-105, state :180-181) */
    KK3_KDA_Q = 0, KK3_KDA_K, KK3_KDA_V, KK3_KDA_OUTPUT_GATE, KK3_KDA_O, KK3_KDA_FA, KK3_KDA_FB, KK3_KDA_BETA,
    KK3_KDA_ONORM, KK3_KDA_A_LOG, KK3_KDA_DT_BIAS, KK3_KDA_CONV_WEIGHT, KK3_KDA_CONV_STATE, KK3_KDA_RECURRENT_STATE,
    /* gated MLA attention (kimi.py:93-97, caches :177-178); shares slot numbers with KDA */
    KK3_MLA_QA = 0, KK3_MLA_QB, KK3_MLA_KA, KK3_MLA_KB, KK3_MLA_O, KK3_MLA_OUTPUT_GATE, KK3_MLA_QN, KK3_MLA_KN,
    KK3_MLA_KV_CACHE, KK3_MLA_PE_CACHE,
    /* dense FFN (kimi.py:106-109) */
    KK3_DENSE_GATE = 16, KK3_DENSE_UP, KK3_DENSE_DOWN,
    /* latent MoE (kimi.py:110-121) */
    KK3_MOE_LATENT_DOWN = 16, KK3_MOE_LATENT_UP, KK3_MOE_LATENT_NORM, KK3_MOE_ROUTER, KK3_MOE_ROUTER_BIAS,
    KK3_MOE_GATE_BLOCKS, KK3_MOE_GATE_SCALES, KK3_MOE_UP_BLOCKS, KK3_MOE_UP_SCALES, KK3_MOE_DOWN_BLOCKS,
    KK3_MOE_DOWN_SCALES, KK3_MOE_SHARED_GATE, KK3_MOE_SHARED_UP, KK3_MOE_SHARED_DOWN,
    KK3_LAYER_SLOTS = 32
};

/* Number of pointer-table slots for a geometry: KK3_GLOBAL_SLOTS + layers * KK3_LAYER_SLOTS. */
int kk3_table_size(const kk3_config* cfg);

/* Check a pointer table against a geometry on the host only (no CUDA call): KK3_OK, or KK3_ERR_ARG when its
 * size is wrong, a used slot is NULL or a pointer is misaligned; the step entry points make the same checks
 * before launching. */
int kk3_check_table(const kk3_config* cfg, const void* const* table, int table_size);

/* Create a context: validate the geometry, allocate device scratch and the symmetric exchange buffer.
 * Replaces the reference's per-rank set-up inside `build(case)` (megabench/harness/runner.py:53-69,
 * harness/distributed.py:67-77). Returns KK3_OK and *out, or a negative code. */
int kk3_init(const kk3_config* cfg, kk3_ctx** out);

/* tp > 1: export this rank's exchange buffer as a CUDA IPC handle (64 bytes), to be all-gathered over the
 * reference's tp_group (harness/distributed.py:67-69 hands it to build()). */
int kk3_ipc_handle(kk3_ctx* ctx, void* handle64);

/* tp > 1: map every peer's exchange buffer; `handles` holds tp handles of 64 bytes in tp_rank order
 * (this rank's own entry is ignored). Replaces the NCCL all-reduces of kimi.py:343-347 and :218-227,
 * which then run inside the step kernel as one-shot NVLink peer stores. */
int kk3_open_peers(kk3_ctx* ctx, const void* handles);

/* Enqueue one decode step on `stream` (a cudaStream_t; NULL = legacy default stream). Asynchronous:
 * one cooperative kernel launch, no allocation, no copies. Replaces `run(inputs)`
 * (megabench/harness/runner.py:66-69) / `kimi.reference` (kimi.py:230-340) for this rank. */
int kk3_step(kk3_ctx* ctx, const void* const* table, int table_size, void* stream);

/* Multi-step decoding with in-place cache append (no counterpart in the reference's per-step API; the
 * reference's own tools chain steps by feeding the outputs back as the next step's state,
 * tools/verify_kimi_vs_hf.py:145-154). Same table, math and outputs as kk3_step, except:
 *  - `lengths` (device int64 [batch], 8-byte aligned) gives each row's number of cached MLA positions; the row
 *    attends positions [0, lengths[b]) of its cache plus the new token (only the new token after a reset), and
 *    every lengths[b] must be below the context the context was created with (the cache capacity);
 *  - each MLA layer's new latent and rope entries are also written into that layer's kv_cache / pe_cache input
 *    at position lengths[b] (0 after a reset): the cache inputs are updated in place;
 *  - cache_length = lengths[b] + 1 (1 after a reset), so the previous step's cache_length output can be passed
 *    as the next step's `lengths`, even as the same buffer;
 *  - the KDA state outputs may alias the state inputs (each layer's input a view of the stacked output tensor):
 *    every state element is read before it is written, by the same thread.
 * A row whose length is at or beyond the capacity makes the step fail (status KK3_ERR_DEVICE). */
int kk3_step_append(kk3_ctx* ctx, const void* const* table, int table_size, const int64_t* lengths, void* stream);

/* Device-side status of the most recent steps, read from mapped host memory without synchronising:
 * KK3_OK, KK3_ERR_TIMEOUT or KK3_ERR_DEVICE. Call after the stream has been synchronised. A step that fails
 * also writes next_token = -1 and cache_length = 0 into its outputs, and every later kk3_step on the context
 * returns KK3_ERR_FAILED. */
int kk3_status(kk3_ctx* ctx);

/* Allocation-free variant of kk3_init + kk3_step + kk3_free for one TP1 step (no counterpart in the
 * reference). For callers that cannot allocate device memory when they run a step: serving engines that have
 * already handed nearly all of HBM to their own caches and pool, and latency-bound loops that must not call
 * cudaMalloc/cudaFree, which synchronise the device. The step's scratch is a file-scope device array of
 * 32 MiB per device; nothing is allocated. Geometries whose scratch does not fit get KK3_ERR_TOO_LARGE,
 * tp > 1 gets KK3_ERR_UNSUPPORTED (a static device symbol cannot be exported to peers over CUDA IPC).
 * The first call on a device does set-up (symbol address, kernel attributes); make it before any stream
 * capture containing this call. Each call enqueues two device operations on `stream`: a cudaMemsetAsync of the
 * scratch words that must start at zero (the whole planned scratch when the geometry differs from the previous
 * call's on this device), then the step's cooperative launch. `error_word` (optional, a device-accessible int
 * the caller zeroed) is set to a nonzero device code if an in-kernel wait times out. With error_word = NULL
 * a failed step is visible only in its outputs (next_token = -1, cache_length = 0, as every failed step
 * writes them), and the next call clears the internal error state: there is no status query. Calls whose
 * steps overlap on one device share the scratch and race: serialise them. Same table, outputs and
 * arithmetic as kk3_step. */
int kk3_step_noalloc(const kk3_config* cfg, const void* const* table, int table_size, void* stream,
                     int* error_word);

/* Human-readable text for a return code. */
const char* kk3_error_string(int code);

/* Release everything kk3_init / kk3_open_peers acquired. */
void kk3_free(kk3_ctx* ctx);

/* --- diagnostics (not used by run()) ------------------------------------------------------------- */

/* Like kk3_step, but the kernel returns after `stop_phase` grid-wide phases (stop_phase < 0: all). */
int kk3_debug_step(kk3_ctx* ctx, const void* const* table, int table_size, void* stream, int stop_phase);

/* Run only phases [start_phase, stop_phase) (stop_phase < 0: to the end); earlier phases are skipped
 * entirely, so their scratch results must already be in place (e.g. from a previous full step). Used to
 * time and profile one phase in isolation. */
int kk3_debug_phases(kk3_ctx* ctx, const void* const* table, int table_size, void* stream, int start_phase,
                     int stop_phase);

/* Number of grid-wide phases one step runs (known after the first step). */
int kk3_phase_count(kk3_ctx* ctx);

/* Device address and size of an internal scratch buffer (ids in kk3_debug_buffer_id). */
enum kk3_debug_buffer_id {
    KK3_BUF_PREFIX = 0, KK3_BUF_XA, KK3_BUF_XM, KK3_BUF_ATTN_IN, KK3_BUF_SCORES, KK3_BUF_LATENT,
    KK3_BUF_SHARED_ACT, KK3_BUF_X3, KK3_BUF_ROUTE_W, KK3_BUF_QKV, KK3_BUF_MLA_Q, KK3_BUF_ABSORBED,
    KK3_BUF_ATTN_LAT, KK3_BUF_EXPERT_SUM, KK3_BUF_BLOCKS, KK3_BUF_EXCHANGE,
    KK3_BUF_PHASE_TS, /* u64 globaltimer (ns) at kernel start and at the end of every grid phase */
    KK3_BUF_ARRIVE_TS, /* u64 [256 phases][grid] barrier arrival time of every CTA */
    KK3_BUF_SUB_TS,    /* u64 [256 phases][16] sub-phase stamps of one CTA or warp */
    KK3_BUF_WARP_TS,   /* u64 [256 phases][grid][16 warps] time each GEMV / expert engine warp finished */
    KK3_BUF_COUNT
};
int kk3_debug_buffer(kk3_ctx* ctx, int id, void** ptr, size_t* bytes);

/* Synchronous device-to-device copy of the first `bytes` bytes of a scratch buffer into `dst`. */
int kk3_debug_copy(kk3_ctx* ctx, int id, void* dst, size_t bytes);

/* Bytes of this rank's exchange buffer (flags + two parity regions). */
size_t kk3_exchange_bytes(kk3_ctx* ctx);

/* Byte offsets inside this rank's exchange buffer (8 values): the flag array [B][tp] u32, the two parity data
 * regions, the bytes of one region, and inside a region the sub-regions att bf16 [tp][hidden/16][bp][16],
 * exp f32 [tp][B][latent_hidden], shd bf16 [tp][hidden/16][bp][16], key u64 [tp][B]. bp is the batch padded to
 * 8, 16, 32 or 64 (the kernel's n-tile width); channel ch of batch row b is element
 * ((ch / 16) * bp + b) * 16 + ch % 16 of a source's slot, so that one 16-channel tile of a source is contiguous. */
int kk3_exchange_layout(kk3_ctx* ctx, long long* offsets);

/* Exchange transport of the tensor-parallel reductions (kimi.py:343-347, :218-227).
 * KK3_COMM_PEER (default, the product): one-shot peer stores and release flags inside the one launch.
 * KK3_COMM_HOST (comparison baseline, no counterpart in the reference's API): each rank writes its partial only
 * into its own slot of its own buffer and never waits; the MoE combine and argmax phases each split in two
 * (write, then read). The caller runs the step as phase ranges with kk3_debug_phases and reduces the slots with
 * NCCL between them: all-reduce (FP32 sum) of this rank's att, exp and shd slots, all-gather of the keys.
 * KK3_COMM_PUSH (in-kernel alternative, one launch): the projections' partials (att, shd) are stored only into
 * this rank's own slot; at the start of the phase that reads them every CTA copies its 1/G share of that slot to
 * every peer in 16-byte pieces and raises one release flag per (source, CTA). The routed-expert sums, the
 * embedding rows and the argmax keys go as with KK3_COMM_PEER. */
#define KK3_COMM_PEER 0
#define KK3_COMM_HOST 1
#define KK3_COMM_PUSH 2
int kk3_set_comm_mode(kk3_ctx* ctx, int mode);

/* The engine of the BF16 projections. KK3_GEMV_AUTO (the default): tcgen05.mma kind::f16 on the tensor cores
 * (M = 128 weight rows, N = the batch padded to 32 or 64, FP32 accumulators in TMEM) for batches above 16, the
 * warp-level mma.sync engine for batches up to 16. KK3_GEMV_MMA: mma.sync for every batch (the comparison
 * engine). Both sum in FP32; results may differ in the last bit of a rounded value. No counterpart in the
 * reference. Takes effect at the next step. */
#define KK3_GEMV_AUTO 0
#define KK3_GEMV_MMA 1
int kk3_set_gemv_engine(kk3_ctx* ctx, int engine);

/* Single-process testing aid: use an existing device allocation of kk3_exchange_bytes() bytes as rank r's
 * exchange buffer instead of an IPC mapping (no counterpart in the reference). */
int kk3_debug_set_peer(kk3_ctx* ctx, int r, void* device_ptr);

/* Fault localisation: enable (1) or disable (0) per-CTA progress publishing to mapped host memory, and copy
 * the current words (2 x 1024 ints: [0][cta] = phase reached, [1][cta] = progress code) into `out` (may be
 * NULL). Readable after a device fault, when the context can no longer be queried. */
int kk3_debug_trace(kk3_ctx* ctx, int enable, int* out, int n);

/* Launch shape of the step kernel: CTAs (one per SM), threads per CTA, dynamic shared memory bytes. */
int kk3_launch_config(kk3_ctx* ctx, int* grid, int* threads, size_t* smem);

#ifdef __cplusplus
}
#endif

#endif /* KK3_H */
