/* chalot_b200.h — C ABI of the B200 (sm_100a) implementation of chalot_C1's
 * sparse-MoE decode hot path.
 *
 * Every entry point returns an int status (CHALOT_OK or a negative code); the
 * message of the last failure on the calling thread is chalot_last_error().
 * Nothing aborts the process. Engine handles are single-threaded, as the
 * reference's `&mut self` Engine is.
 *
 * Reference interfaces replaced (paths within chalot28/chalot_C1):
 *   Engine::load             src/model/engine.rs:94
 *   Engine::forward          src/model/engine.rs:173
 *   Engine::generate         src/model/engine.rs:497
 *   Engine::sample_from_logits src/model/engine.rs:551
 *   InferenceState::logits   src/model/state.rs:20
 *   matmul_int8              src/tensor/matmul.rs:47
 *   matmul_int4              src/tensor/matmul.rs:363
 *   quantize_f32_to_i8       src/tensor/quantization.rs:26
 *   softmax_top_k (router)   src/tensor/normalization.rs:203, engine.rs:334-344
 *   PagedKVCache             src/model/memory.rs:100-201
 */
#ifndef CHALOT_B200_H
#define CHALOT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CHALOT_OK 0
#define CHALOT_ERR_ARG (-1)     /* bad argument or unsupported shape */
#define CHALOT_ERR_IO (-2)      /* file open/read/write failed */
#define CHALOT_ERR_FORMAT (-3)  /* bad magic/version/size in a .myai file */
#define CHALOT_ERR_OOM (-4)     /* device or host allocation failed */
#define CHALOT_ERR_CUDA (-5)    /* a CUDA runtime call failed */
#define CHALOT_ERR_NCCL (-6)    /* an NCCL call failed */
#define CHALOT_ERR_TIMEOUT (-7) /* a bounded wait ran out */
#define CHALOT_ERR_STATE (-8)   /* call not valid in the handle's state */

/* ---- library ---------------------------------------------------------- */

/* Message of the last failed call on this thread ("" if none). */
const char* chalot_last_error(void);
/* ABI version: major*10000 + minor*100 + patch. */
int chalot_abi_version(void);
/* Device-side checks of the asynchronous operators (a bounded wait of the
 * tensor-core MoE path or of the paged attention that gave up, a page id
 * outside a paged pool) are recorded on the device and returned by the next
 * operator call on that device once the failing work has finished
 * (CHALOT_ERR_TIMEOUT or CHALOT_ERR_ARG), with no synchronisation inside the
 * calls. This call synchronises `stream` and returns such a status at once
 * (CHALOT_OK if none); the record is cleared when reported. No reference
 * counterpart: the reference's ops are synchronous and panic
 * (src/tensor/matmul.rs:47-54 asserts; src/model/memory.rs:76-84 writes). */
int chalot_device_status(void* stream);

/* ---- .myai writer (host only) ----------------------------------------- */

/* Shape and seed of a synthetic model. Weights are N(0, weight_std) and are
 * quantized as the reference's quantizers do (int8 per-tensor absmax for
 * embeddings/attention/lm_head, int4 per-row-per-group absmax/7 for experts). */
typedef struct chalot_synth_spec {
  uint32_t dim, hidden_dim, n_layers, n_heads, vocab_size;
  uint32_t n_experts, top_k, int4_group_size, max_seq_len;
  uint32_t rope_theta_x100; /* header field: theta*100, 0 = 10000 */
  float weight_std;         /* 0 selects 0.02 */
  uint64_t seed;
  int n_threads; /* <= 0: all hardware threads; the output does not depend on it */
} chalot_synth_spec;

/* Writes a .myai v2 file. No counterpart in the reference's Rust API; its
 * layout is the one src/model/dummy.rs:17 and qwen_to_myai.py write. */
int chalot_myai_write_synthetic(const char* path, const chalot_synth_spec* spec);

/* Header-derived configuration of a .myai file (src/model/config.rs:40-69). */
typedef struct chalot_model_config {
  uint32_t dim, hidden_dim, n_layers, n_heads, head_dim, vocab_size, max_seq_len;
  uint32_t n_experts, top_k, int4_group_size, depth_router_layer;
  float rope_theta;
  uint64_t total_bytes;        /* WeightIndex::total_bytes */
  uint64_t expert_bytes;       /* bytes of one expert (gate+up+down, with scales) */
} chalot_model_config;

/* Parses the header of a file and computes its size (host only). */
int chalot_myai_inspect(const char* path, chalot_model_config* out);

/* Checks a whole .myai file (host only): magic, version, flag bits, that the
 * reserved bytes 32-127 of a v2 header are zero (train_distill.py:898-915
 * writes the v2 fields there, packed after the v1 ones), the shape, and the
 * exact size implied by the header (validate_myai.py:99-129 only estimates it
 * within a factor of two). Returns CHALOT_OK or CHALOT_ERR_FORMAT; `report`
 * (may be NULL) receives one "error: ..." or "note: ..." line per finding. */
int chalot_myai_validate(const char* path, char* report, size_t cap);

/* ---- engine ----------------------------------------------------------- */

typedef struct chalot_engine chalot_engine;

typedef struct chalot_opts {
  int device;          /* CUDA device ordinal */
  int use_cuda_graph;  /* 1: replay one captured graph per forward (default) */
} chalot_opts;

typedef enum chalot_strategy {
  CHALOT_GREEDY = 0,
  CHALOT_TOP_K = 1,
  CHALOT_TOP_P = 2,
  CHALOT_MIN_P = 3
} chalot_strategy;

/* Mirrors SamplingConfig (src/model/engine.rs:37-62). */
typedef struct chalot_sampling {
  int strategy;
  float temperature;
  uint32_t top_k;
  float top_p;
  float min_p;
  float repetition_penalty; /* applied when > 1 (engine.rs:555) */
  uint32_t repetition_window;
  const uint32_t* stop_tokens;
  uint32_t n_stop_tokens;
  /* Seed of the draws of the TOP_K / TOP_P / MIN_P strategies (splitmix64,
   * one draw per sampled token). 0 seeds from the clock, as the reference's
   * random_f32 (src/tensor/sampling.rs:15-30) does. */
  uint64_t seed;
} chalot_sampling;

/* Engine::load: parse the header, upload the weights to the device, build
 * the RoPE tables and the KV cache. `opts` may be NULL. */
int chalot_load(const char* path, const chalot_opts* opts, chalot_engine** out);
void chalot_free(chalot_engine* e);
int chalot_get_config(const chalot_engine* e, chalot_model_config* out);

/* Engine::forward: one token at position `pos`; writes the argmax token.
 * The logits stay on the device until chalot_get_logits. */
int chalot_forward(chalot_engine* e, uint32_t token, uint32_t pos, uint32_t* out_token);

/* Engine::generate: prefill `prompt` token by token, then decode up to
 * `max_new` tokens. `out` must hold `max_new` entries; *n_out receives the
 * count written. `sampling` NULL means greedy with no repetition penalty. */
int chalot_generate(chalot_engine* e, const uint32_t* prompt, size_t n_prompt,
                    size_t max_new, const chalot_sampling* sampling,
                    uint32_t* out, size_t* n_out);

/* Engine::sample_from_logits over the logits of the last forward, with the
 * repetition penalty applied to `history` (the last repetition_window ids). */
int chalot_sample_from_logits(chalot_engine* e, const chalot_sampling* sampling,
                              const uint32_t* history, size_t n_history,
                              uint32_t* out_token);

/* One token from device logits [V] with the strategy of `cfg` (its penalty,
 * window and stop tokens are ignored) for the uniform draw r in [0, 1):
 * sample_argmax / sample_top_k / sample_top_p / sample_min_p
 * (src/tensor/sampling.rs:34-165). The logits are not modified. Synchronous;
 * *out_token receives the token. */
int chalot_sample(const float* logits, size_t vocab, const chalot_sampling* cfg, float r,
                  uint32_t* out_token, void* stream);

/* Copies the logits of the last forward (state.logits) to host memory. */
int chalot_get_logits(chalot_engine* e, float* dst, size_t n);

/* ---- batched decode --------------------------------------------------- */
/* Several sequences through one engine, one token each per call. The
 * reference runs one Engine per sequence (Engine::forward, engine.rs:173,
 * has no batch); here each sequence owns a KV cache slot and a call advances
 * n of them at once with the same per-token arithmetic, so every sequence
 * decodes exactly as it would alone. MoE models only. */

/* Allocates max_seqs KV cache slots (f32, [slot][layer][max_seq_len][dim])
 * and the batch buffers; once per engine. */
int chalot_batch_reserve(chalot_engine* e, uint32_t max_seqs);

/* Engine::forward for n rows: token toks[i] at position pos[i] of the
 * sequence in slot slots[i]; writes each row's argmax token. A slot may appear
 * in several rows at distinct positions: every row's K/V is written before
 * any row attends, so rows p, p+1, ... of one sequence run as consecutive
 * forwards would (a prompt in one pass, or the k draft tokens of speculative
 * decoding verified at once; Engine::forward has no batch, engine.rs:173). */
int chalot_forward_batch(chalot_engine* e, const uint32_t* slots, const uint32_t* toks,
                         const uint32_t* pos, uint32_t n, uint32_t* out_toks);

/* Logits of row `row` (the i-th token) of the last chalot_forward_batch. */
int chalot_get_batch_logits(chalot_engine* e, uint32_t row, float* dst, size_t n);

/* chalot_batch_reserve with a paged K/V cache, the batch counterpart of the
 * reference's PagedKVCache (src/model/memory.rs:119-185): f32 rows (so every
 * sequence still decodes exactly as alone) in a pool of n_pages pages of
 * page_tokens positions (a power of two in [16, 256]), page p holding
 * [layer][position][dim] for K and for V. A slot takes pages from the pool as
 * chalot_forward_batch writes its positions (CHALOT_ERR_OOM when none is
 * left) and returns them with chalot_batch_release, so the cache holds the
 * positions in use rather than max_seqs x max_seq_len. head_dim % 16 == 0. */
int chalot_batch_reserve_paged(chalot_engine* e, uint32_t max_seqs, uint32_t n_pages, uint32_t page_tokens);

/* Returns a slot's K/V pages to the pool (paged reserve; a no-op for the flat
 * cache). The slot's next sequence starts at position 0. */
int chalot_batch_release(chalot_engine* e, uint32_t slot);

/* The reserve's max_seqs (0 before chalot_batch_reserve). */
int chalot_batch_capacity(chalot_engine* e, uint32_t* max_seqs);

/* Pool state of a paged reserve: free pages, all pages, positions per page
 * (all 0 for the flat cache). Any pointer may be NULL. */
int chalot_batch_kv_pages(chalot_engine* e, uint32_t* n_free, uint32_t* n_total, uint32_t* page_tokens);

/* ---- continuous batching ------------------------------------------------ */
/* A scheduler over chalot_forward_batch (the reference serves one prompt at a
 * time, engine.rs:497-548): sequences are submitted at any time; each
 * chalot_sched_step admits waiting sequences into free slots (with a paged
 * reserve, only when the pool holds pages for their prompt + max_new
 * positions beside those the running sequences may still take), gives every
 * decoding sequence one row and the prefilling ones chunks of their prompt
 * with the rows left (up to max_rows per forward), runs one forward, and
 * retires sequences that produced max_new tokens or a stop token (the stop
 * token is not returned, as in chalot_generate), releasing their slot and
 * pages. Decoding is greedy; every sequence's tokens are those of
 * chalot_generate on its prompt alone. One engine, no expert-parallel group. */
typedef struct chalot_sched chalot_sched;

/* The engine must be reserved (chalot_batch_reserve or _paged); max_rows in
 * [1, its max_seqs]; slots are the engine's max_seqs slots. */
int chalot_sched_create(chalot_engine* e, uint32_t max_rows, chalot_sched** out);
void chalot_sched_free(chalot_sched* s);

/* Queues a prompt (n >= 1 tokens) for max_new >= 1 greedy tokens, ending
 * early at any of the n_stop stop tokens; n + max_new - 1 <= max_seq_len.
 * *id identifies it in chalot_sched_poll. */
int chalot_sched_submit(chalot_sched* s, const uint32_t* prompt, size_t n, uint32_t max_new, const uint32_t* stop,
                        size_t n_stop, uint64_t* id);

/* One forward over the running sequences (none: nothing runs). Any output
 * pointer may be NULL: sequences running and waiting after the step, rows in
 * the forward. */
int chalot_sched_step(chalot_sched* s, uint32_t* n_running, uint32_t* n_waiting, uint32_t* n_rows);

/* Tokens a sequence has produced so far (up to cap of them into out; *n_out
 * the total) and whether it is done. A done sequence is forgotten after a poll
 * that returns all of its tokens. CHALOT_ERR_ARG for an unknown id. */
int chalot_sched_poll(chalot_sched* s, uint64_t id, uint32_t* out, size_t cap, size_t* n_out, int* done);

/* Measured peak of the int8 tensor cores on the current device: one CTA per
 * SM streams `iters` x 4 tcgen05.mma.kind::i8 M128 x N256 x K32 out of shared
 * memory; *tops = int8 TOP/s (2 ops per multiply-add), *ms = kernel time.
 * The denominator of the MoE prefill's tensor roofline; no counterpart in the
 * reference. */
int chalot_probe_int8_mma(int iters, double* tops, double* ms);

/* Self-check of the library's exact float division (the kernels divide with a
 * fused-multiply-add correction of a reciprocal approximation instead of the
 * compiler's slower sequence, and must round exactly as IEEE division): n
 * pseudo-random pairs from `seed` plus pairs in the ranges the decode path
 * divides; *mismatches receives the count of bitwise differences from the
 * compiler's division, example[0..1] (may be NULL) one mismatching pair. No
 * reference counterpart (device arithmetic check). */
int chalot_selftest_division(uint64_t n, uint64_t seed, uint64_t* mismatches, float* example);

/* ---- expert parallelism of the batched forward ---------------------------- */
/* The reference runs one process; these spread the expert block of
 * Engine::forward (engine.rs:353-401) over a group of engines, one per GPU:
 * expert e is computed by rank e % world, attention and the other dense parts
 * by every rank for its own sequences. Per MoE layer chalot_forward_batch then
 * routes its tokens, sends each (token, choice) row (int8, exact) to the
 * expert's rank, runs its local experts on the rows it received, sends the
 * f32 outputs back and combines them in selection order, so every sequence
 * decodes exactly as on one GPU. All ranks must reserve the same max_seqs and
 * call chalot_forward_batch the same number of times (n = 0 allowed: the rank
 * still takes part in the exchanges). Waits on peers are bounded
 * (CHALOT_ERR_TIMEOUT). */

/* A 128-byte NCCL unique id, made on rank 0 and passed to the others out of
 * band (e.g. torch.distributed). */
int chalot_ep_nccl_id(uint8_t* id);
/* Joins the group `id` as `rank` of `world` over NCCL on the engine's device
 * (world divides n_experts). */
int chalot_ep_attach_nccl(chalot_engine* e, uint32_t rank, uint32_t world, const uint8_t* id);

/* In-process group: engines of one process (one per thread) exchange through
 * a hub; several may share a GPU. For tests of the distributed path. */
typedef struct chalot_ep_hub chalot_ep_hub;
chalot_ep_hub* chalot_ep_hub_create(uint32_t world);
void chalot_ep_hub_free(chalot_ep_hub* hub);
int chalot_ep_attach_hub(chalot_engine* e, chalot_ep_hub* hub, uint32_t rank);

/* Leaves the group (the engine computes every expert again). */
int chalot_ep_detach(chalot_engine* e);

/* Device time of the prefill and decode phases of the last chalot_generate,
 * measured with CUDA events on the engine's stream, and the forward counts.
 * After a chalot_forward_batch: its device time as decode_ms, its rows as
 * n_decode, prefill 0. */
int chalot_last_timing(chalot_engine* e, double* prefill_ms, double* decode_ms,
                       uint32_t* n_prefill, uint32_t* n_decode);

/* Expert path of every layer at batch 1 (routing + gate/up + down of the
 * top_k experts the router picks from the engine's current residual, on a
 * private copy of it), captured once and replayed `reps` times: mean device
 * time per layer and the expert weight bytes one layer streams. */
int chalot_bench_moe_layers(chalot_engine* e, int reps, double* ms_per_layer,
                            double* bytes_per_layer);

/* Phase timestamps of the last decode step when the engine runs the
 * persistent one-kernel step (the shapes it fits; CHALOT_DECODE=kernels at
 * load selects the multi-kernel chain, for which this returns
 * CHALOT_ERR_STATE): %globaltimer ns seen by CTA 0, [n_layers + 1][16]; per
 * layer 0 start, 1 attention input (after the grid barrier), 2 QKV done,
 * 3 scores start, 4 scores done, 5 softmax/PV start, 6 PV done, 7 O start,
 * 8 O done, 9 routing start, 10 expert copies issued, 11 gate/up done,
 * 12 down start, 13 down done; then the kernel's start, lm_head start and
 * lm_head end. *n_out receives the element count. No reference counterpart
 * (measurement of the engine.rs:213-401 layer loop on the device). */
int chalot_decode_trace(chalot_engine* e, unsigned long long* dst, size_t n, size_t* n_out);

/* Device time of every kernel of one forward (token, pos), in launch order:
 * embed, then per layer qkv, attention scores, attention softmax.PV, O
 * projection (+ routing), gate/up, down; then lm_head. Runs the forward twice
 * from a graph with an event after each kernel (no programmatic overlap) and
 * reports the second run. *n_out = 1 + 6*n_layers + 1. */
int chalot_profile_forward(chalot_engine* e, uint32_t token, uint32_t pos, float* ms, int cap,
                           int* n_out);

/* ---- operators (device pointers, caller-owned memory) ------------------- */
/* `stream` is a cudaStream_t (NULL = the legacy default stream). The input
 * vector is quantized on the device exactly as quantize_f32_to_i8 does. */

/* matmul_int8: out[r] = ((float)dot_i32(w[r,:], q(x)) * w_scales[r]) * x_scale. */
int chalot_matmul_i8(float* out, const int8_t* w, const float* w_scales, const float* x,
                     size_t out_dim, size_t in_dim, void* stream);

/* matmul_int4: per row, t += ((float)gdot_g * s[r,g]) * x_scale in group order;
 * w_packed is [out_dim][ceil(in_dim/2)] (low nibble = even column, value-8),
 * w_scales is [out_dim][ceil(in_dim/group)]. group 0 selects 64. */
int chalot_matmul_i4(float* out, const uint8_t* w_packed, const float* w_scales,
                     const float* x, size_t out_dim, size_t in_dim, size_t group,
                     void* stream);

/* quantize_f32_to_i8 for n_vec vectors of length n: q[v,:] and scale[v]. */
int chalot_quantize_i8(int8_t* q, float* scale, const float* x, size_t n_vec, size_t n,
                       void* stream);

/* Router of one MoE layer for n_tok tokens (engine.rs:334-344):
 * logits[t,e] = b[e] + dot_f32(w[e,:], x[t,:]); softmax_top_k(logits[t], k).
 * Writes idx[t,k] (int32) and weight[t,k] (f32), in descending weight order. */
int chalot_router_topk(int32_t* idx, float* weight, const float* x, const float* w,
                       const float* b, size_t n_tok, size_t dim, size_t n_experts,
                       size_t top_k, void* stream);

/* ---- batched MoE layer (device pointers, caller-owned memory) ----------- */

/* One MoE FFN layer as a .myai file stores it (src/model/weight_index.rs:
 * 126-160): router W [E][dim] f32 and b [E] f32, then E experts back to back,
 * each {gate+up packed int4 [2*hidden][dim/2] (gate rows first), their scales
 * [2*hidden][dim/group] f32, down packed [dim][hidden/2], scales
 * [dim][hidden/group]}. `experts` must be 16-byte aligned. group 0 selects 32. */
typedef struct chalot_moe_desc {
  uint32_t dim, hidden_dim, n_experts, top_k, group;
  const float* router_w;
  const float* router_b;
  const uint8_t* experts;
} chalot_moe_desc;

/* Bytes of device workspace chalot_moe_layer needs for n_tok tokens (0 when
 * the descriptor is invalid; chalot_last_error says why). */
size_t chalot_moe_workspace_size(const chalot_moe_desc* desc, size_t n_tok);

/* The expert block of Engine::forward (src/model/engine.rs:334-401) for n_tok
 * input rows x[n_tok][dim] that are already the FFN's normalised input:
 * router logits, softmax_top_k, then per selected expert gate/up matmul_int4,
 * swiglu, down matmul_int4, and out[t] = 0 + w_0*y_0 + w_1*y_1 ... in
 * selection order (the residual add is the caller's). Bit-exact with the
 * reference's per-token arithmetic. sel_out/selw_out ([n_tok][top_k], may be
 * NULL) receive the router's choices. `workspace` (256-byte aligned, at least
 * chalot_moe_workspace_size bytes) is scratch owned by the caller; calls that
 * share it must not overlap. Asynchronous on `stream`; a tensor-core wait
 * that gave up is reported by the next operator call or chalot_device_status
 * (CHALOT_ERR_TIMEOUT). */
int chalot_moe_layer(const chalot_moe_desc* desc, const float* x, size_t n_tok, float* out,
                     int32_t* sel_out, float* selw_out, void* workspace,
                     size_t workspace_bytes, void* stream);

/* chalot_moe_layer without a workspace argument. This entry point has no
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they run a layer, such as a host whose own allocator
 * owns the device's whole memory budget, or a host binding only plain
 * pointers through an FFI. Its scratch is a fixed 4 MiB array inside the
 * library on each device (held by every GPU that loads the library until the
 * process exits); calls needing more scratch than that on the path it runs
 * (the tile-GEMM path; e.g. more than 73 tokens at dim 896, hidden 4864,
 * top-2) fail with CHALOT_ERR_ARG. It allocates nothing. The first call on a
 * device looks up the array's device address, so make that call before any
 * stream capture on the device; the address is kept, so do not use this
 * entry point across a cudaDeviceReset. All calls on a device share the
 * array: calls that overlap on the GPU (other streams or threads without
 * ordering) race. Output matches chalot_moe_layer's bit for bit. */
int chalot_moe_layer_noalloc(const chalot_moe_desc* desc, const float* x, size_t n_tok,
                             float* out, int32_t* sel_out, float* selw_out, void* stream);

/* ---- expert-parallel MoE layer in one call ------------------------------ */
/* Expert e lives on rank e % world, one rank per GPU of one node with NVLink
 * peer access. Each rank exports an exchange arena in its GPU memory; the
 * ranks move int8 token rows to the experts and f32 outputs back with plain
 * peer stores (counts and offsets stay on the device: no host round trip, no
 * padding on the wire) and the layer is bit-identical to chalot_moe_layer on
 * one GPU. It replaces the parallel region of the reference's expert block,
 * the rayon par_iter over the selected experts (src/model/engine.rs:353-387),
 * with expert parallelism across GPUs. */
#define CHALOT_EP_HANDLE_BYTES 64
typedef struct chalot_ep_comm chalot_ep_comm;

/* This rank's side of a group of `world` ranks (<= 8) for layers shaped like
 * `desc` (its experts pointer is ignored here) and calls of up to max_tokens
 * tokens, on the current device. `handle` receives CHALOT_EP_HANDLE_BYTES
 * bytes that the other ranks need to reach this rank's arena; all-gather the
 * handles over any host transport (rank order) and pass them to
 * chalot_ep_comm_connect. */
int chalot_ep_comm_create(uint32_t rank, uint32_t world, const chalot_moe_desc* desc, size_t max_tokens,
                          chalot_ep_comm** out, uint8_t* handle);
/* Maps every other rank's arena (all_handles: world x CHALOT_EP_HANDLE_BYTES). */
int chalot_ep_comm_connect(chalot_ep_comm* comm, const uint8_t* all_handles);
void chalot_ep_comm_free(chalot_ep_comm* comm);

/* The expert block (as chalot_moe_layer) for this rank's n_tok rows, with the
 * experts spread over the group: desc holds the full router (n_experts = all
 * experts) and in `experts` only this rank's experts e (e % world == rank),
 * in increasing e, each in the file layout. Every rank of the group must call
 * it, the same number of times and in the same order (n_tok may be 0); a rank
 * that does not arrive makes the others report CHALOT_ERR_TIMEOUT (bounded
 * device waits). Asynchronous on `stream`. */
int chalot_moe_layer_ep(chalot_ep_comm* comm, const chalot_moe_desc* desc, const float* x, size_t n_tok,
                        float* out, int32_t* sel_out, float* selw_out, void* stream);

/* ---- expert-parallel MoE layer: building blocks ------------------------- */
/* Expert e lives on rank e % n_ranks. Per layer each rank routes its tokens,
 * plans and gathers its (token, choice) slots by destination, exchanges
 * counts, int8 rows and scales with the other ranks (the caller's NCCL
 * all-to-all), runs chalot_moe_experts on the rows it received, sends the
 * outputs back and combines them. Together: the expert block of
 * Engine::forward (src/model/engine.rs:334-401), bit-identical to
 * chalot_moe_layer. All pointers are device memory; all calls are
 * asynchronous on `stream`. */

/* Router, softmax_top_k and quantize_f32_to_i8 of n_tok rows:
 * sel/selw [n_tok][top_k], xq [n_tok][dim] int8, xs [n_tok]. */
int chalot_moe_route(const chalot_moe_desc* desc, const float* x, size_t n_tok, int32_t* sel,
                     float* selw, int8_t* xq, float* xs, void* stream);

/* Stable order of the n_slots slots (sel flattened) by (rank, local expert):
 * order[p] = slot at position p, pos[slot] = its position (-1 for an expert id
 * outside [0, n_experts)), offsets[n_experts + 1] = position where the key
 * (rank, local expert) = rank * (n_experts / n_ranks) + local starts. */
int chalot_moe_plan(const int32_t* sel, size_t n_slots, uint32_t n_experts, uint32_t n_ranks,
                    int32_t* order, int32_t* pos, int32_t* offsets, void* stream);

/* rows[p] = xq[order[p] / top_k], row_scales[p] = xs[order[p] / top_k];
 * dim % 16 == 0, 16-byte aligned rows. */
int chalot_moe_gather(const int8_t* xq, const float* xs, const int32_t* order, size_t n_slots,
                      uint32_t top_k, size_t dim, int8_t* rows, float* row_scales, void* stream);

/* Expert outputs y[i] = down(swiglu(gate(x_i), up(x_i))) of expert
 * row_expert[i] for n_rows already-quantized rows (matmul_int4 on rows[i] with
 * scale row_scales[i], engine.rs:366-380). `local` describes the experts this
 * rank holds (n_experts = its count, router pointers unused). */
size_t chalot_moe_experts_workspace_size(const chalot_moe_desc* local, size_t n_rows);
int chalot_moe_experts(const chalot_moe_desc* local, const int8_t* rows, const float* row_scales,
                       const int32_t* row_expert, size_t n_rows, float* y, void* workspace,
                       size_t workspace_bytes, void* stream);

/* out[t] = 0 + selw[t][0] * y[pos[t*top_k]] + selw[t][1] * y[pos[t*top_k+1]] ...
 * in selection order (slots with pos < 0 are skipped). */
int chalot_moe_combine(const float* y, const int32_t* pos, const float* selw, size_t n_tok,
                       uint32_t top_k, size_t dim, float* out, void* stream);

/* ---- PagedKVCache (the reference's paged KV manager) -------------------- */
/* PagedKVCache (src/model/memory.rs:100-201) with its pages in device memory:
 * 256-token pages per layer, K and V rows int8 with one scale per row
 * (max|x|/127, 1.0 for a zero row; (x/scale).clamp(-128, 127) truncated, as
 * `as i8`), LRU eviction of the least recently written page once the cache
 * holds max_pages_per_layer * n_layers pages (0 selects the reference's 16),
 * checked before every write. Reads leave the LRU order alone. One cache per
 * host thread, as the reference's &mut self. */
typedef struct chalot_kv_cache chalot_kv_cache;

/* PagedKVCache::new(kv_dim, n_layers) (memory.rs:119-127). */
int chalot_kv_create(uint32_t kv_dim, uint32_t n_layers, uint32_t max_pages_per_layer, int device,
                     chalot_kv_cache** out);
void chalot_kv_free(chalot_kv_cache* c);
/* PagedKVCache::write (memory.rs:163-171); k, v: host rows of kv_dim f32. */
int chalot_kv_write(chalot_kv_cache* c, uint32_t layer, uint32_t pos, const float* k, const float* v);
/* PagedKVCache::read (memory.rs:174-185): *found = 0 (outputs untouched) when
 * the page is absent; k_out, v_out: host rows. */
int chalot_kv_read(chalot_kv_cache* c, uint32_t layer, uint32_t pos, float* k_out, float* v_out,
                   int* found);
/* n writes in order, as n calls of chalot_kv_write would leave the cache;
 * pos: host array; k, v: device rows [n][kv_dim]. */
int chalot_kv_write_batch(chalot_kv_cache* c, uint32_t layer, const uint32_t* pos, size_t n,
                          const float* k, const float* v, void* stream);
/* n reads: k_out, v_out device rows [n][kv_dim] (rows whose page is absent are
 * left untouched), found: host array of n flags. */
int chalot_kv_gather(chalot_kv_cache* c, uint32_t layer, const uint32_t* pos, size_t n, float* k_out,
                     float* v_out, uint8_t* found, void* stream);
/* PagedKVCache::clear, active_pages, memory_mb (memory.rs:129-133, 188-201). */
int chalot_kv_clear(chalot_kv_cache* c);
size_t chalot_kv_active_pages(const chalot_kv_cache* c);
float chalot_kv_memory_mb(const chalot_kv_cache* c);

/* ---- paged int8 KV cache for long-context decode ------------------------ */

/* A device page pool in the long-context format (new; the reference's own
 * PagedKVCache, src/model/memory.rs:100-201, keeps 256-token pages with one
 * scale per token row): pages of page_tokens (8, 16 or 32) tokens; the K block
 * and the V block of each head in a page (page_tokens x head_dim values,
 * token-major) are int8 with one f32 scale per block (quantize_f32_to_i8's
 * rule: absmax/127, round to nearest even).
 *   data   [n_pages][2 (K, V)][n_heads][page_tokens][head_dim] int8, 16-B aligned
 *   scales [n_pages][2][n_heads] f32
 * head_dim 64 or 128, n_heads at most 31. Memory is owned by the caller. */
typedef struct chalot_paged_kv {
  uint32_t n_pages, page_tokens, n_heads, head_dim;
  int8_t* data;
  float* scales;
} chalot_paged_kv;

/* Quantizes n whole pages into the pool: k and v are f32
 * [n][page_tokens][n_heads][head_dim] (device), the tokens of page page_ids[i]
 * (device int32) in order. Asynchronous on `stream` (KVPage::write_token,
 * memory.rs:76-84, is synchronous on the host). Out-of-range page ids are
 * skipped on the device and reported by the next operator call or by
 * chalot_device_status (CHALOT_ERR_ARG). */
int chalot_paged_kv_store(const chalot_paged_kv* kv, const int32_t* page_ids, size_t n,
                          const float* k, const float* v, void* stream);

/* Device workspace bytes of chalot_paged_attention (0 on a bad pool). */
size_t chalot_paged_attention_workspace_size(const chalot_paged_kv* kv, size_t n_seq,
                                             size_t max_pages);

/* Decode-step attention of n_seq sequences over the pool: per sequence s and
 * head h, the attention of Engine::forward (src/model/engine.rs:283-309) over
 * the dequantized rows of tokens [0, seq_lens[s]), whose pages are
 * page_table[s][0..] ([n_seq][max_pages] int32, device):
 * s_t = 30*tanh((q.k_t / sqrt(head_dim)) / 30), softmax, out = sum_t p_t v_t.
 * q, out: [n_seq][n_heads][head_dim] f32 (device). Float sums are reordered
 * (split pages, online softmax): agreement is to float tolerance, not bits.
 * Asynchronous; a page id outside the pool is read as page 0 and reported by
 * the next operator call or chalot_device_status (CHALOT_ERR_ARG). */
int chalot_paged_attention(const chalot_paged_kv* kv, const float* q, size_t n_seq,
                           const int32_t* page_table, size_t max_pages, const int32_t* seq_lens,
                           float* out, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CHALOT_B200_H */
