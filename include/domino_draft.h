/*
 * domino_draft.h -- C ABI of libdomino_draft.so, the B200 (sm_100a) draft step
 * of Domino speculative decoding: GRU correction head + correction MLP +
 * lm_head greedy argmax + greedy prefix acceptance.
 *
 * Conventions
 *   - Every pointer argument named "device" is CUDA device memory on the
 *     handle's device; nothing here allocates per call or synchronises.
 *   - Tensors are row-major; "ld" is the row stride in elements.
 *   - Weights are bf16 (DD_BF16) or fp16 (DD_FP16); token ids are int64.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL =
 *     the legacy default stream).  Calls are asynchronous and can be
 *     captured into a CUDA graph as long as the same pointers are replayed.
 *   - Return value: DD_OK (0) or a negative DD_E* status; nothing throws
 *     across the ABI.  dd_last_error() gives a one-line reason.
 *   - A handle belongs to one device and is not thread-safe.
 *
 * Reference interfaces replaced (paths inside the Domino repository):
 *   dd_create + dd_set_weights + dd_build_table
 *       DraftCorrectionGraphRunner.__init__   code/kernel/domino.py:245-372
 *   dd_rollout
 *       DraftCorrectionGraphRunner.__call__   code/kernel/domino.py:495-508
 *       (its captured body _forward_impl      code/kernel/domino.py:374-431)
 *   dd_draft_block
 *       base_logits = target.lm_head(parallel_hiddens) and the pure-draft
 *       prefix argmax, code/dflash.py:424-427, followed by the runner call of
 *       code/dflash.py:429-439
 *   dd_accept
 *       greedy acceptance, code/dflash.py:472-485
 */
#ifndef DOMINO_DRAFT_H
#define DOMINO_DRAFT_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DD_OK 0
#define DD_EINVAL (-1)      /* bad argument: shape, dtype, alignment, null pointer */
#define DD_ECUDA (-2)       /* a CUDA runtime/driver call failed */
#define DD_EDEVICE (-3)     /* a kernel reported an error (status word); see dd_get_status */
#define DD_EUNSUPPORTED (-4) /* device is not sm_100 / feature not built */

#define DD_BF16 0
#define DD_FP16 1
#define DD_F32 2   /* logits only (dd_verify_accept) */

/* Device status bits (dd_get_status). */
#define DD_STATUS_TIMEOUT 1u       /* a bounded wait inside a kernel gave up */
#define DD_STATUS_BAD_TOKEN 2u     /* a token id was outside [0, vocab) and was clamped */
#define DD_STATUS_NO_ARGMAX 4u     /* an argmax saw no candidate at all */

/* Argmax semantics, in every kernel here: the lowest index wins a tie, and a
 * NaN of either sign ranks above every number (the first NaN wins), as
 * torch.argmax does. */

typedef struct dd_handle dd_handle;

/* Shapes of one runner (code/kernel/domino.py:245-256). */
typedef struct dd_config {
  int32_t batch;          /* B: rows per call */
  int32_t steps;          /* S: draft tokens produced by one rollout */
  int32_t hidden;         /* H: target hidden size (fc1 takes H+G inputs) */
  int32_t gru_hidden;     /* G: GRU state size */
  int32_t emb_dim;        /* E: correction-MLP width (fc1 outputs) */
  int32_t vocab;          /* V */
  int32_t prefix_tokens;  /* 1 + pure_draft_prefix_len */
  int32_t dtype;          /* DD_BF16 or DD_FP16 */
} dd_config;

/* Non-owning device pointers to the head's parameters, in the reference's
 * layouts (code/kernel/domino.py:272-327; code/dflash.py:261-274).  The
 * pointed-to memory must outlive the handle or the next dd_set_weights. */
typedef struct dd_weights {
  const void* fc1;       int64_t fc1_ld;      /* [E, H+G]: W_z = fc1[:, :H], W_s = fc1[:, H:] */
  const void* fc1_bias;                       /* [E] or NULL */
  const void* fc2;       int64_t fc2_ld;      /* [V, E] */
  const void* fc2_bias;                       /* [V] or NULL */
  const void* w_hh;      int64_t w_hh_ld;     /* [3G, G], gate order (r, z, n) */
  const void* b_hh;                           /* [3G] or NULL */
  const void* table;     int64_t table_ld;    /* [V, 3G] = embed @ W_ih^T + b_ih (dd_build_table) */
  const void* lm_head;   int64_t lm_head_ld;  /* [V, H] or NULL; needed by dd_draft_block only */
} dd_weights;

/* Create a handle for `device` (allocates the handle's scratch once). */
int dd_create(const dd_config* cfg, int device, dd_handle** out);

/* Point the handle at the head's weights and prepare their TMA descriptors.
 * With the packed layout (dd_set_weight_layout) it also copies W_z, W_s,
 * W_hh, fc2 and lm_head once into handle-owned buffers of 16 KB tiles in the
 * order the tensor cores read them (one extra copy of those matrices in HBM;
 * it synchronises the device).  Call again after the weights change. */
int dd_set_weights(dd_handle* h, const dd_weights* w);

/* How dd_rollout / dd_draft_block run the rollout after the z projection:
 * 0 one persistent cooperative kernel for all prefix and draft steps when the
 * handle allows it (unsharded, at most 64 phases), else one kernel per phase;
 * 1 (default) always one kernel per phase, measured 1-5 % faster on B200.
 * DD_ROLLOUT_PERSISTENT=1 in the environment selects 0 at dd_create.  Both
 * give identical tokens. */
int dd_set_rollout_mode(dd_handle* h, int mode);

/* The middle of the correction MLP, embed_proj = (Linear, middle, Linear)
 * (code/kernel/domino.py:15-50).  DD_MIDDLE_SILU (default) is the reference's
 * fused path: SiLU(z + s) in fp32 into an fp32 fc2 contraction (domino.py:58-136).
 * For any other middle the reference runs its PyTorch branch
 * (domino.py:406-431), and so does this library: mid = middle(z + s), the fc2
 * logits and base + logits, and every op of the GRU cell (with tanh) rounded
 * to the weight dtype.  DD_MIDDLE_SILU_ROUNDED is a SiLU the reference does not
 * fuse (a middle of several modules, e.g. SiLU then Dropout). */
#define DD_MIDDLE_SILU 0
#define DD_MIDDLE_IDENTITY 1
#define DD_MIDDLE_RELU 2
#define DD_MIDDLE_GELU 3       /* erf form */
#define DD_MIDDLE_GELU_TANH 4  /* tanh approximation */
#define DD_MIDDLE_TANH 5
#define DD_MIDDLE_SIGMOID 6
#define DD_MIDDLE_SILU_ROUNDED 7
int dd_set_middle(dd_handle* h, int middle);

/* packed = 0 (default: stream the caller's row-major weights in place, no
 * extra memory) or 1 (stream the packed copy with 1-D bulk copies; measured
 * equal speed at the default launch shape; DD_PACK_WEIGHTS=1 in the
 * environment selects it at dd_create).  Takes effect at the next
 * dd_set_weights. */
int dd_set_weight_layout(dd_handle* h, int packed);

/* table[v, :] = embed[v, :] @ W_ih^T + b_ih, rounded to the weight dtype
 * (code/kernel/domino.py:322-327).  embed [V, H], w_ih [3G, H], b_ih [3G] or
 * NULL, table_out [V, 3G] with row stride 3G. */
int dd_build_table(dd_handle* h, const void* embed, int64_t embed_ld, const void* w_ih,
                   int64_t w_ih_ld, const void* b_ih, void* table_out, void* stream);

/* One rollout: the runner call of code/kernel/domino.py:495-508.
 *   prefix_ids       [B, prefix_tokens] int64 (verify_ids[:, :1+p])
 *   parallel_hiddens [B, S, H]                (hidden states of the S positions)
 *   base_logits      [B, S, V]                (target.lm_head of those positions)
 *   out_tokens       [B, S] int64             (greedy corrected draft tokens) */
int dd_rollout(dd_handle* h, const int64_t* prefix_ids, const void* parallel_hiddens,
               const void* base_logits, int64_t* out_tokens, void* stream);

/* The whole draft side of one block (code/dflash.py:424-439) with the lm_head
 * projection fused in: base = lm_head(parallel_hiddens) for all K = p + S
 * positions, the p pure-draft prefix tokens = argmax(base[:, :p]), then the
 * rollout over positions p..K-1.
 *   last_token       [B] int64     (verify_ids[:, 0], the last accepted token)
 *   parallel_hiddens [B, K, H]
 *   base_logits_out  [B, K, V]     (written; bf16/fp16 like the weights)
 *   verify_out       [B, K + 1] int64: (last_token, p prefix tokens, S draft tokens) */
int dd_draft_block(dd_handle* h, const int64_t* last_token, const void* parallel_hiddens,
                   void* base_logits_out, int64_t* verify_out, void* stream);

/* dd_rollout for callers that cannot allocate device memory (no counterpart
 * in the reference).  Some callers cannot call cudaMalloc: code running while
 * a CUDA graph is captured, hosts whose own pool owns all of HBM and treat any
 * other allocation as a leak, and stateless foreign-function bindings with no
 * place to keep a handle's buffers between calls.  This entry point takes the
 * same inputs and outputs as dd_rollout plus the config, the weights and the
 * device, and allocates nothing: its scratch is a 32 MiB static device array
 * inside the library, which every GPU that loads the library holds until the
 * process exits.
 *   - The first call on a device looks up that array's device address; make
 *     it before any stream capture on that device.
 *   - Shapes whose scratch exceeds 32 MiB are rejected with DD_EINVAL and a
 *     message (at H = G = 4096, E = 12288, V = 151936, 15 steps on 148 SMs:
 *     batch <= 6).
 *   - All calls share the one array and it keeps the last call's contents;
 *     the call clears what must start at zero.  Calls whose work overlaps on
 *     the GPU (two streams, or two host threads on one device) race on it:
 *     order them on one stream.
 *   - Host-side errors are returned at once, with a reason in
 *     dd_last_error(NULL).  What the kernels find while running (a bounded
 *     wait that gave up, a clamped token id) collects in a status word of
 *     the same static array: read it with dd_noalloc_status. */
int dd_rollout_noalloc(const dd_config* cfg, const dd_weights* w, int device, const int64_t* prefix_ids,
                       const void* parallel_hiddens, const void* base_logits, int64_t* out_tokens,
                       void* stream);

/* Status of the allocation-free calls on `device` (no counterpart in the
 * reference): waits for the device, then returns and clears the DD_STATUS_*
 * bits that dd_rollout_noalloc's kernels have set since the last read (0 =
 * every call ran clean; 0 as well when no such call has run).  Negative on a
 * CUDA error.  A caller without a handle has no dd_get_status; this is the
 * one way it learns that a rollout timed out (DD_STATUS_TIMEOUT: discard its
 * tokens) or that a prefix id was out of range.  It allocates nothing. */
int dd_noalloc_status(int device);

/* Greedy acceptance (code/dflash.py:472-485) for every row:
 *   verify_ids [B, K1] int64, posterior [B, K1] int64 (K1 = draft tokens + 1)
 *   accept_out [B] int32: leading draft tokens equal to the target's
 *   bonus_out  [B] int64: posterior[b, accept_out[b]]
 * The reference records accept + 1 as the block's acceptance length. */
int dd_accept(const int64_t* verify_ids, const int64_t* posterior, int32_t batch, int32_t k1,
              int32_t* accept_out, int64_t* bonus_out, void* stream);

/* ---- Vocab sharding across GPUs (one process per GPU) --------------------
 * Each rank owns vocab rows [vocab_begin, vocab_end) of fc2 and lm_head and
 * replicates the rest; per draft step every rank computes its (logit, index)
 * argmax word and the fc2 kernel that finishes it writes it straight into
 * every rank's exchange buffer over NVLink (peer stores), after which the
 * next kernel on each rank takes the maximum over ranks: an all-reduce(max)
 * of packed (logit, index) words, fused into the kernels (no separate
 * collective).
 * The s / gh projections (W_s, W_hh) are split by 128-row slices too: each
 * rank computes its slice, raises a flag in every rank's buffer, and a small
 * gather kernel copies the other ranks' slices in over NVLink.
 *
 * Setup per rank: dd_create -> dd_get_exchange_buffer -> dd_ipc_export ->
 * (exchange the 64-byte handles between processes, e.g. all_gather) ->
 * dd_ipc_open of every other rank's handle -> dd_set_vocab_shard ->
 * dd_set_weights with fc2 / lm_head (/ fc2_bias) pointing at this rank's
 * rows.  dd_rollout's base_logits stay full-vocab rows; dd_draft_block
 * writes only this rank's columns ([B, K, vocab_end - vocab_begin]). */

/* This handle's exchange buffer (device memory, for dd_ipc_export). */
int dd_get_exchange_buffer(dd_handle* h, void** dev_ptr, uint64_t* bytes);

/* cudaIpcGetMemHandle of a device allocation; handle_out receives 64 bytes. */
int dd_ipc_export(const void* dev_ptr, void* handle_out);

/* Map another process's exported allocation on `device`; close with dd_ipc_close. */
int dd_ipc_open(int device, const void* handle_in, void** dev_ptr_out);
int dd_ipc_close(int device, void* dev_ptr);

/* Make this handle rank `rank` of `world` (<= 8) with vocab rows
 * [vocab_begin, vocab_end); peer_exchange_buffers[j] is rank j's exchange
 * buffer as mapped in this process (entry `rank` is ignored).  Must be
 * followed by dd_set_weights.  world = 1 restores the unsharded handle. */
int dd_set_vocab_shard(dd_handle* h, int32_t rank, int32_t world, int64_t vocab_begin, int64_t vocab_end,
                       void* const* peer_exchange_buffers);

/* Limit of the bounded wait for the other ranks' argmax words (default 2 s);
 * when it runs out the step uses the words that arrived and the status word
 * gets DD_STATUS_TIMEOUT. */
int dd_set_exchange_timeout(dd_handle* h, uint64_t timeout_ns);

/* The target-side half of code/dflash.py:472-485 fused into one pass:
 * posterior[b, j] = argmax_v target_logits[b, j, v] (lowest index on ties and
 * NaN above every number, as torch.argmax) and the greedy acceptance of
 * verify_ids against it; the
 * [B, k1, V] logits are read once and no intermediate is written.
 *   target_logits [B, k1, V] (DD_BF16, DD_FP16 or DD_F32), V = cfg.vocab
 *   verify_ids [B, k1] int64; posterior_out [B, k1] int64;
 *   accept_out [B] int32 (accepted draft tokens); bonus_out [B] int64.
 * k1 <= 64.  Calls on one handle must not overlap on the GPU. */
int dd_verify_accept(dd_handle* h, const void* target_logits, int32_t logits_dtype, int32_t k1,
                     const int64_t* verify_ids, int64_t* posterior_out, int32_t* accept_out,
                     int64_t* bonus_out, void* stream);

/* Debugging and parity aid (no counterpart in the reference): the per-step
 * states of the rollout, in the weight dtype, as the kernels compute and use
 * them.  Device buffers; any of them may be NULL.  With P = prefix_tokens
 * (plus the pure-draft prefix positions for dd_draft_block) and S = steps:
 *   z  [B, K, E]          z projection (+ fc1 bias); K = S for dd_rollout,
 *                         p + S for dd_draft_block
 *   h  [P + S - 1, B, G]  GRU state after prefix token j (entries 0..P-1,
 *                         entry P-1 = the state entering draft step 0), then
 *                         after the GRU step of draft step t (entry P + t)
 *   gh [P - 1 + S - 1, B, 3G]  h W_hh^T + b_hh of prefix token j >= 1 (entry
 *                         j - 1), then of draft step t (entry P - 1 + t)
 *   s  [S, B, E]          s projection h W_s^T of draft step t (entry t)
 * The mapping of code/kernel/domino.py:381-431: z = z_part_all, the h entry
 * P - 1 = gru_hidden after the prefix GRU, s = s_proj, gh = the F.linear of
 * line 420 and the h entries >= P = the _fused_gru_cell outputs. */
typedef struct dd_trace {
  void* z;
  void* h;
  void* gh;
  void* s;
} dd_trace;

/* While a trace is set (t != NULL), dd_rollout and dd_draft_block also copy
 * every state above into it, on the call's stream, between their launches
 * (one kernel per phase; the persistent rollout is not used).  NULL stops
 * tracing.  Unsharded handles only.  Slower: for tests and debugging. */
int dd_set_trace(dd_handle* h, const dd_trace* t);

/* Launch kinds reported by dd_read_timing. */
#define DD_PHASE_Z 1      /* z = parallel_hiddens @ W_z^T */
#define DD_PHASE_ZLM 2    /* the same fused with the lm_head base logits */
#define DD_PHASE_GH 3     /* gh = h @ W_hh^T (prefix GRU) */
#define DD_PHASE_SGH 4    /* s = h @ W_s^T -> SiLU mid, and gh = h @ W_hh^T */
#define DD_PHASE_FC2 5    /* fc2 contraction + base logits + argmax */
#define DD_PHASE_TABLE 6  /* embed @ W_ih^T table */
#define DD_PHASE_CELL 7   /* token pick + GRU cell */
#define DD_PHASE_GATHER 8 /* vocab sharding: other ranks' s / gh slices copied in */
#define DD_PHASE_ROLLOUT 9 /* the whole rollout as one persistent kernel */

/* Benchmarking aid (no counterpart in the reference): while enabled, the
 * handle records a CUDA event pair around every kernel it launches on the
 * caller's stream.  The events separate launches that otherwise overlap
 * (programmatic dependent launch), so enable it only to time kernels. */
int dd_set_timing(dd_handle* h, int enable);

/* Synchronise, return the number n of launches recorded since timing was
 * enabled or last read (at most max_records), their DD_PHASE_* kinds and
 * durations in milliseconds, and clear the record. */
int dd_read_timing(dd_handle* h, int32_t* kinds, float* ms, int32_t max_records);

/* Synchronise the handle's device and return (and clear) its status word
 * (DD_STATUS_* bits); negative on a CUDA error.  After DD_STATUS_TIMEOUT the
 * handle's scratch may be inconsistent: destroy it and create a new one. */
int dd_get_status(dd_handle* h);

/* One-line reason for the last failing call on this handle (never NULL). */
const char* dd_last_error(const dd_handle* h);

/* Library version string. */
const char* dd_version(void);

/* Free the handle's scratch; does not touch the weights. */
int dd_destroy(dd_handle* h);

#ifdef __cplusplus
}
#endif

#endif /* DOMINO_DRAFT_H */
