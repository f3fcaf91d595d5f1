/*
 * mf_head.h — C-ABI of the B200 DFA-restricted output head.
 *
 * Every entry point takes plain device pointers with their sizes in bytes,
 * a cudaStream_t passed as `void*`, and returns an mf_status whose `code`
 * uses the numbering of the reference's marketforge::ErrorCode
 * (include/marketforge/core/status.hpp:7-31), so a C++ wrapper converts it
 * to marketforge::Status by a cast.  All launches are asynchronous on the
 * given stream; arguments are validated on the host before any launch, in
 * the reference's order (src/cuda/greedy.cu:349-399):
 *   zero dims / zero maximum / null stream        -> MF_INVALID_ARGUMENT
 *   vocab or maximum > UINT32_MAX, rows > INT_MAX -> MF_RESOURCE_LIMIT
 *   a size product overflowing uint64             -> MF_ARITHMETIC_OVERFLOW
 *   a byte size that does not match exactly, a null or aliased buffer
 *                                                 -> MF_INVALID_ARGUMENT
 *   a buffer not aligned to its widest element (2-byte halves, 4-byte
 *   ints and scores, 8-byte keys and workspace; cudaMalloc memory always
 *   is)                                           -> MF_INVALID_ARGUMENT
 *   the launch failing                            -> MF_CUDA_BACKEND_FAILURE,
 *                                                    detail = cudaError_t
 * Bad rows found on the device produce MF_INVALID_TOKEN, never a trap.
 *
 * Selection rule shared by every head/select entry point: the highest FP32
 * score wins, equal scores resolve to the lowest token id, NaN never wins,
 * and a valid row whose every score is NaN selects its lowest candidate id.
 */
#ifndef MF_HEAD_H
#define MF_HEAD_H

#include <stdint.h>

#if defined(__GNUC__)
#define MF_API __attribute__((visibility("default")))
#else
#define MF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* marketforge::ErrorCode values used here (status.hpp:7-31). */
enum {
  MF_OK = 0,
  MF_INVALID_ARGUMENT = 1,
  MF_ARITHMETIC_OVERFLOW = 5,
  MF_RESOURCE_LIMIT = 15,
  MF_CUDA_BACKEND_FAILURE = 21,
  MF_CUDA_RUNTIME_FAILURE = 22
};

/* marketforge::Status (status.hpp:33-49) as a C struct. */
typedef struct mf_status {
  int32_t code;
  uint32_t detail;
} mf_status;

/* restricted_greedy_invalid_token_id (include/marketforge/cuda/greedy.hpp:11-12). */
#define MF_INVALID_TOKEN 0xFFFFFFFFu

/* Library version and the device architecture it was built for (1000 = sm_100a). */
MF_API uint32_t mf_version(void);
MF_API uint32_t mf_built_arch(void);

/* ---- reference-signature entry points ----------------------------------- */

/* Replaces marketforge::cuda::greedy_select_f16
 * (include/marketforge/cuda/greedy.hpp:17-21, src/cuda/greedy.cu:237-279).
 * logits: fp16 [rows, vocab]; token_ids: u32 [rows].  All-NaN rows select 0. */
MF_API mf_status mf_greedy_select_f16(const void* logits, uint64_t logits_bytes,
                               void* token_ids, uint64_t token_ids_bytes,
                               uint64_t rows, uint64_t vocab, void* stream);

/* Replaces marketforge::cuda::restricted_greedy_select_f16
 * (greedy.hpp:29-33, greedy.cu:281-347).  allowed: u32 [rows, max_allowed],
 * counts: u32 [rows].  count 0, count > max_allowed or a candidate >= vocab
 * gives MF_INVALID_TOKEN for that row. */
MF_API mf_status mf_restricted_greedy_select_f16(const void* logits, uint64_t logits_bytes,
                                          const void* allowed, uint64_t allowed_bytes,
                                          const void* counts, uint64_t counts_bytes,
                                          void* token_ids, uint64_t token_ids_bytes,
                                          uint64_t rows, uint64_t vocab,
                                          uint64_t max_allowed, void* stream);

/* Replaces marketforge::cuda::restricted_output_head_f16
 * (greedy.hpp:43-49, greedy.cu:349-414): the fused gather-GEMV + argmax over
 * a padded candidate table.  hidden: fp16 [rows, hidden_size]; embedding:
 * fp16 [vocab, hidden_size]; allowed: u32 [rows, max_allowed]; counts: u32
 * [rows]; token_ids: u32 [rows].  Needs no workspace: each row is owned by
 * one thread block. */
MF_API mf_status mf_restricted_output_head_f16(const void* hidden, uint64_t hidden_bytes,
                                        const void* embedding, uint64_t embedding_bytes,
                                        const void* allowed, uint64_t allowed_bytes,
                                        const void* counts, uint64_t counts_bytes,
                                        void* token_ids, uint64_t token_ids_bytes,
                                        uint64_t rows, uint64_t hidden_size,
                                        uint64_t vocab, uint64_t max_allowed,
                                        void* stream);

/* ---- ragged CSR head (new batched launch path) --------------------------
 *
 * Row r's candidates are ids[offsets[r] .. offsets[r+1]) (i32), the flat
 * form the callers built as a padded table from TokenDfa::allowed
 * (src/tools/cuda_restricted_greedy_bench.cu:107-165).  The candidates of
 * the whole batch are split evenly over the GPU, so one long row is shared
 * by many thread blocks; partial results merge through 64-bit atomic max on
 * a packed (score, id) key in `workspace`, which makes the result
 * independent of scheduling.  A call is the head kernel on `stream`, and, for
 * batches of up to 4,096 rows that span more than one thread block, a small
 * second kernel that decodes the row keys into out_ids / out_scores and
 * clears them.
 *
 * workspace: mf_head_workspace_bytes(rows) bytes of device memory, zero-filled
 * once by the caller before its first use; every call leaves it zero again.
 * Calls that share a workspace must not overlap on the GPU.
 * out_ids: u32 [rows]; out_scores: f32 [rows] or NULL (the winning FP32 score,
 * NaN for all-NaN or invalid rows).  Empty rows and rows with a candidate
 * outside [0, vocab) give MF_INVALID_TOKEN.  If the offsets are malformed
 * (offsets[0] != 0, decreasing, or offsets[rows] != total_ids) every row gives
 * MF_INVALID_TOKEN; the kernel never reads outside ids[0, total_ids). */
MF_API uint64_t mf_head_workspace_bytes(uint64_t rows);

MF_API mf_status mf_head_restricted_csr_f16(const void* hidden, uint64_t hidden_bytes,
                                     const void* embedding, uint64_t embedding_bytes,
                                     const void* offsets, uint64_t offsets_bytes,
                                     const void* ids, uint64_t ids_bytes,
                                     void* out_ids, uint64_t out_ids_bytes,
                                     void* out_scores, uint64_t out_scores_bytes,
                                     void* workspace, uint64_t workspace_bytes,
                                     uint64_t rows, uint64_t hidden_size,
                                     uint64_t vocab, void* stream);

/* mf_head_restricted_csr_f16 with launch options.  MF_LAUNCH_OVERLAP_PREVIOUS:
 * the launch may begin while the previous kernel on `stream` is still running
 * (programmatic dependent launch), so back-to-back batches overlap one's
 * tail with the next one's gathers.  The head waits for the previous
 * kernel before its first write (workspace, outputs), but reads hidden,
 * offsets, ids and the embedding without waiting: use the flag only when the
 * previous kernel on the stream does not write them (e.g. consecutive head
 * calls on independent batches).  Any other bit is invalid_argument. */
#define MF_LAUNCH_OVERLAP_PREVIOUS 1u
MF_API mf_status mf_head_restricted_csr_f16_ex(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t rows, uint64_t hidden_size,
    uint64_t vocab, uint32_t launch_flags, void* stream);

/* mf_head_restricted_csr_f16_ex with the candidate ids as u16 [total_ids]
 * (ids_bytes = 2 * total_ids), for vocabularies of at most 65,536 ids
 * (invalid_argument otherwise; SmolLM2's is 49,152): half the bytes for a
 * caller that moves batches from host memory.  Results are those of the
 * int32 entry on the same ids.  No counterpart in the reference, whose ids
 * are int32 (include/marketforge/cuda/greedy.hpp). */
MF_API mf_status mf_head_restricted_csr_u16ids_f16_ex(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t rows, uint64_t hidden_size,
    uint64_t vocab, uint32_t launch_flags, void* stream);

/* The same head with the decoder's final RMSNorm fused in front: `hidden`
 * holds the last layer's un-normalised rows (fp16 [rows, hidden_size]) and
 * gamma the norm weight (fp16 [hidden_size], 16-byte aligned).  Each row is
 * normalised in registers as rms_norm_f16 (src/cuda/rms_norm.cu:69-100)
 * followed by the head would see it: inv = 1 / sqrt(mean(x^2) + eps) in
 * FP32, h = fp16(x * inv * w).  Replaces the rms_norm_f16 launch before
 * restricted_output_head_f16 (src/cuda/smollm2.cu:474-492).  eps must be
 * finite and > 0 (rms_norm_f32's rule, src/cpu/operators.cpp:498-501). */
MF_API mf_status mf_head_restricted_csr_rmsnorm_f16(
    const void* hidden, uint64_t hidden_bytes, const void* gamma, uint64_t gamma_bytes, float eps,
    const void* embedding, uint64_t embedding_bytes, const void* offsets, uint64_t offsets_bytes,
    const void* ids, uint64_t ids_bytes, void* out_ids, uint64_t out_ids_bytes, void* out_scores,
    uint64_t out_scores_bytes, void* workspace, uint64_t workspace_bytes, uint64_t rows,
    uint64_t hidden_size, uint64_t vocab, void* stream);

/* ---- device-resident DFA: allowed-set lookup + head + advance ------------
 *
 * The DFA is CSR over states, the flat form of TokenDfa/ActionDfa's
 * StateRecord{first_arc, arc_count} + GrammarArc{token, next}
 * (include/marketforge/grammar/token_dfa.hpp:54-58, action_dfa.hpp:20-27):
 * state s allows tokens arc_tokens[state_offsets[s] .. state_offsets[s+1])
 * (sorted ascending, as TokenDfa::build emits them) and taking the k-th arc
 * moves to arc_next[k].  One step: for each sequence b, look up the allowed
 * set of states_in[b], run the restricted head on hidden[b], write the
 * chosen token to out_tokens[b] and the next state to states_out[b]
 * (TokenDfa::advance, src/grammar/token_dfa.cpp:111-128).  A sequence whose
 * state is out of range or has no arcs gets MF_INVALID_TOKEN and keeps its
 * state.  The workspace rule is the same as for the CSR head: one step needs
 * mf_head_workspace_bytes(batch) bytes, mf_dfa_decode_f16 needs
 * mf_dfa_workspace_bytes(batch) (three more 8-byte words per sequence: with a
 * vocabulary of at most 65,536 ids and fewer than 65,535 states, a step hands
 * its results to the next through rotating key buffers instead of per-row
 * arrival counters). */
MF_API uint64_t mf_dfa_workspace_bytes(uint64_t batch);

MF_API mf_status mf_dfa_head_step_f16(const void* hidden, uint64_t hidden_bytes,
                               const void* embedding, uint64_t embedding_bytes,
                               const void* state_offsets, uint64_t state_offsets_bytes,
                               const void* arc_tokens, uint64_t arc_tokens_bytes,
                               const void* arc_next, uint64_t arc_next_bytes,
                               const void* states_in, uint64_t states_in_bytes,
                               void* states_out, uint64_t states_out_bytes,
                               void* out_tokens, uint64_t out_tokens_bytes,
                               void* out_scores, uint64_t out_scores_bytes,
                               void* workspace, uint64_t workspace_bytes,
                               uint64_t batch, uint64_t num_states, uint64_t hidden_size,
                               uint64_t vocab, void* stream);

/* mf_dfa_head_step_f16 with the decoder's final RMSNorm fused in front, as
 * mf_head_restricted_csr_rmsnorm_f16: hidden holds the last layer's
 * un-normalised rows, gamma the norm weight (fp16 [hidden_size], 16-byte
 * aligned), eps finite and > 0.  One launch for rms_norm_f16 + the grammar's
 * allowed-set lookup + the head + the DFA advance. */
MF_API mf_status mf_dfa_head_step_rmsnorm_f16(
    const void* hidden, uint64_t hidden_bytes, const void* gamma, uint64_t gamma_bytes, float eps,
    const void* embedding, uint64_t embedding_bytes, const void* state_offsets,
    uint64_t state_offsets_bytes, const void* arc_tokens, uint64_t arc_tokens_bytes,
    const void* arc_next, uint64_t arc_next_bytes, const void* states_in,
    uint64_t states_in_bytes, void* states_out, uint64_t states_out_bytes, void* out_tokens,
    uint64_t out_tokens_bytes, void* out_scores, uint64_t out_scores_bytes, void* workspace,
    uint64_t workspace_bytes, uint64_t batch, uint64_t num_states, uint64_t hidden_size,
    uint64_t vocab, void* stream);

/* `steps` DFA head steps back to back on one stream with no host
 * synchronisation: hidden is fp16 [steps, batch, hidden_size];
 * state_trace is u32 [steps + 1, batch] with row 0 holding the initial
 * states; token_trace is u32 [steps, batch]; score_trace f32 [steps, batch]
 * or NULL.  Step s reads state_trace[s] and writes state_trace[s + 1]. */
MF_API mf_status mf_dfa_decode_f16(const void* hidden, uint64_t hidden_bytes,
                            const void* embedding, uint64_t embedding_bytes,
                            const void* state_offsets, uint64_t state_offsets_bytes,
                            const void* arc_tokens, uint64_t arc_tokens_bytes,
                            const void* arc_next, uint64_t arc_next_bytes,
                            void* state_trace, uint64_t state_trace_bytes,
                            void* token_trace, uint64_t token_trace_bytes,
                            void* score_trace, uint64_t score_trace_bytes,
                            void* workspace, uint64_t workspace_bytes,
                            uint64_t steps, uint64_t batch, uint64_t num_states,
                            uint64_t hidden_size, uint64_t vocab, void* stream);

/* ---- dense full-vocabulary head (tcgen05) --------------------------------
 *
 * Replaces linear_f16 (cuBLAS logits, include/marketforge/cuda/linear.hpp:18-22,
 * src/cuda/linear.cu:40-104) followed by greedy_select_f16 (greedy.hpp:17-21):
 * one kernel computes FP32 scores of every vocabulary row of a shard with
 * the tensor cores and keeps only each row's best (score, id).  hidden: fp16
 * [rows, hidden_size]; embedding: fp16 [vocab_rows, hidden_size], the rows
 * of vocabulary ids [vocab_begin, vocab_begin + vocab_rows).  hidden_size is
 * a multiple of 64 up to 576; rows <= 256 x (SM pairs that can be co-resident).  Outputs (either may
 * be NULL, not both): out_keys u64 [rows] — the packed key whose unsigned
 * max over shards is the global selection (so vocabulary shards on several
 * GPUs merge with one max all-reduce, then mf_decode_keys) — and out_ids u32
 * [rows] / out_scores f32 [rows] for this shard.  A row whose scores are all
 * NaN selects vocab_begin (greedy_select_f16's "token 0" rule per shard).
 * Workspace rule as for mf_head_restricted_csr_f16, sized by
 * mf_dense_workspace_bytes(rows). */
MF_API uint64_t mf_dense_workspace_bytes(uint64_t rows);

MF_API mf_status mf_dense_head_f16(const void* hidden, uint64_t hidden_bytes,
                                   const void* embedding, uint64_t embedding_bytes,
                                   void* out_keys, uint64_t out_keys_bytes,
                                   void* out_ids, uint64_t out_ids_bytes,
                                   void* out_scores, uint64_t out_scores_bytes,
                                   void* workspace, uint64_t workspace_bytes,
                                   uint64_t rows, uint64_t hidden_size,
                                   uint64_t vocab_rows, uint64_t vocab_begin, void* stream);

/* mf_dense_head_f16 with launch options (MF_LAUNCH_OVERLAP_PREVIOUS, declared
 * with mf_head_restricted_csr_f16_ex): the launch may start while the
 * previous kernel on `stream` drains; it reads hidden and embedding without
 * waiting and waits before its first write, so the previous kernel must not
 * write hidden or embedding. */
MF_API mf_status mf_dense_head_f16_ex(const void* hidden, uint64_t hidden_bytes,
                                      const void* embedding, uint64_t embedding_bytes,
                                      void* out_keys, uint64_t out_keys_bytes, void* out_ids,
                                      uint64_t out_ids_bytes, void* out_scores,
                                      uint64_t out_scores_bytes, void* workspace,
                                      uint64_t workspace_bytes, uint64_t rows,
                                      uint64_t hidden_size, uint64_t vocab_rows,
                                      uint64_t vocab_begin, uint32_t launch_flags, void* stream);

/* Decodes packed keys (e.g. after a max all-reduce across vocabulary shards)
 * to ids u32 [rows] and, if out_scores is not NULL, FP32 scores. */
MF_API mf_status mf_decode_keys(const void* keys, uint64_t keys_bytes, void* out_ids,
                                uint64_t out_ids_bytes, void* out_scores,
                                uint64_t out_scores_bytes, uint64_t rows, void* stream);

/* ---- vocabulary shards on several GPUs, merged inside the dense kernel ----
 *
 * Replaces "mf_dense_head_f16 per shard + max all-reduce of the keys +
 * mf_decode_keys" (the reference's single-GPU linear_f16 + greedy_select_f16,
 * src/cuda/linear.cu:40-104 and src/cuda/greedy.cu:237-279, split by vocab
 * rows) with one launch per rank: the kernel's last CTA stores its keys into
 * every rank's exchange buffer over NVLink, raises the rank's flag there,
 * waits (bounded, 100 ms) for every rank's flag for this call, and writes
 * the global ids/scores (and merged keys) on every rank.  One process per GPU, one exchange buffer per
 * rank:
 *   mf_exchange_alloc      cudaMalloc + zero + cudaIpcGetMemHandle (64-byte handle)
 *   (the caller all-gathers the handles, e.g. over torch.distributed)
 *   mf_exchange_open_peer  cudaIpcOpenMemHandle of a peer's handle
 * exchange[q] is rank q's buffer as mapped in this process (the own buffer
 * at exchange[rank]); world <= 8; every rank calls with the same rows, in
 * the same order, on its own GPU.
 * Failure signal: the call returns MF_OK once launched; a rank whose peers
 * do not arrive within 100 ms, or whose peer reports a failed part, gives
 * every row MF_INVALID_TOKEN (sentinel rows are the device-side failure
 * signal) and marks its exchange buffer broken; every later call on a
 * broken buffer gives the sentinel as well (mf_exchange_broken reads the
 * mark) until the caller makes new exchange buffers.  The context stays
 * usable.  launch_flags as for mf_dense_head_f16_ex. */
#define MF_IPC_HANDLE_BYTES 64
MF_API uint64_t mf_exchange_bytes(uint64_t rows, uint32_t world);
MF_API mf_status mf_exchange_alloc(void** buffer, uint64_t bytes, void* ipc_handle);
MF_API mf_status mf_exchange_free(void* buffer);
MF_API mf_status mf_exchange_open_peer(const void* ipc_handle, void** peer_buffer);
MF_API mf_status mf_exchange_close_peer(void* peer_buffer);
/* 1 in *broken once this rank's exchange buffer (its own, as allocated) is
 * marked broken, else 0.  Synchronous 4-byte read. */
MF_API mf_status mf_exchange_broken(const void* buffer, uint32_t* broken);
MF_API mf_status mf_dense_head_sharded_f16(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    void* out_keys, uint64_t out_keys_bytes, void* out_ids, uint64_t out_ids_bytes,
    void* out_scores, uint64_t out_scores_bytes, void* workspace, uint64_t workspace_bytes,
    uint64_t rows, uint64_t hidden_size, uint64_t vocab_rows, uint64_t vocab_begin,
    void* const* exchange, uint64_t exchange_bytes, uint32_t world, uint32_t rank,
    uint32_t launch_flags, void* stream);

/* Self-test of the dense kernel's bounded waits (no counterpart in the
 * reference): a tiny dense problem whose loads are never issued, so its
 * mbarrier waits run out after 100 ms; on return *error_word is 1 and
 * *invalid_rows is 128 when the kernel gave up cleanly.  Synchronises. */
MF_API mf_status mf_dense_selftest_wait_timeout(void* stream, uint32_t* error_word,
                                                uint32_t* invalid_rows);

/* ---- host pipeline for the ragged head ----------------------------------
 *
 * No counterpart in the reference (the reference copies each decode step's
 * inputs and synchronises, src/cuda/smollm2.cu:395-501).  A pipeline owns
 * `depth` slots, each with a stream, device buffers and its own head
 * workspace.  mf_pipeline_submit copies one batch (hidden fp16 [rows,
 * hidden_size], CSR offsets int32 [rows + 1], ids int32 [total_ids]) from
 * host memory to the next slot, runs the ragged head and copies ids (u32
 * [rows]) and scores (f32 [rows], may be NULL) back into the caller's host
 * buffers, all asynchronously on that slot's stream; batches on different
 * slots overlap.  Host buffers should be pinned (a pageable buffer makes its
 * copy synchronous) and must stay untouched until mf_pipeline_wait(ticket)
 * returns.  The embedding stays resident on the device.  mf_pipeline_create
 * allocates the slots (device memory) once. */
typedef struct mf_pipeline mf_pipeline;

MF_API mf_status mf_pipeline_create(mf_pipeline** pipeline, const void* embedding,
                                    uint64_t embedding_bytes, uint64_t vocab,
                                    uint64_t hidden_size, uint64_t max_rows, uint64_t max_ids,
                                    uint32_t depth);
MF_API mf_status mf_pipeline_submit(mf_pipeline* pipeline, const void* hidden, uint64_t rows,
                                    const void* offsets, const void* ids, uint64_t total_ids,
                                    void* out_ids, void* out_scores, uint64_t* ticket);
/* One batch as a single packed host buffer: hidden fp16 [rows, hidden_size],
 * then offsets int32 [rows + 1], then ids int32 [total_ids], back to back
 * (batch_bytes must equal rows*hidden_size*2 + (rows+1)*4 + total_ids*4);
 * `out` receives ids u32 [rows] then scores f32 [rows].  One copy each way
 * instead of up to five. */
MF_API mf_status mf_pipeline_submit_packed(mf_pipeline* pipeline, const void* batch,
                                           uint64_t batch_bytes, uint64_t rows,
                                           uint64_t total_ids, void* out, uint64_t* ticket);
/* mf_pipeline_submit_packed with the ids as u16 [total_ids] (batch_bytes =
 * rows*hidden_size*2 + (rows+1)*4 + total_ids*2), for vocabularies of at most
 * 65,536 ids (invalid_argument otherwise): a batch's ids are most of its
 * bytes, and the host-to-device copy bounds the pipeline.  No counterpart in
 * the reference, whose ids are int32 (include/marketforge/cuda/greedy.hpp). */
MF_API mf_status mf_pipeline_submit_packed_u16ids(mf_pipeline* pipeline, const void* batch,
                                                  uint64_t batch_bytes, uint64_t rows,
                                                  uint64_t total_ids, void* out,
                                                  uint64_t* ticket);
MF_API mf_status mf_pipeline_wait(mf_pipeline* pipeline, uint64_t ticket);
MF_API mf_status mf_pipeline_synchronize(mf_pipeline* pipeline);
/* The number of slots, and slot `slot`'s stream (NULL past the last slot). */
MF_API uint32_t mf_pipeline_depth(mf_pipeline* pipeline);
MF_API void* mf_pipeline_stream(mf_pipeline* pipeline, uint32_t slot);
MF_API void mf_pipeline_destroy(mf_pipeline* pipeline);

/* ---- allocation-free ragged head ----------------------------------------
 *
 * No counterpart in the reference.  The same ragged CSR head as
 * mf_head_restricted_csr_f16, for callers that cannot allocate device
 * memory (code running where cudaMalloc is forbidden or unavailable: inside
 * a host callback, under an allocator that must not grow, or an embedding
 * runtime that hands out only its own input/output buffers).  Its scratch is
 * a fixed array of MF_NOALLOC_SCRATCH_BYTES in this library's device memory,
 * held by every GPU that loads the library until the process exits; rows is
 * limited to MF_NOALLOC_MAX_ROWS (larger batches get MF_RESOURCE_LIMIT).
 * The first call on each device looks the array up (cudaGetSymbolAddress),
 * so make that first call before any stream capture.  Each call clears the
 * part of the array it uses (cudaMemsetAsync on `stream`) and calls no
 * allocator.  All calls on a device share the one array: calls that overlap
 * on the GPU (different streams, no ordering between them) race and give
 * wrong results, so serialise them.  Arguments and results are otherwise
 * those of mf_head_restricted_csr_f16. */
#define MF_NOALLOC_MAX_ROWS 65536u
#define MF_NOALLOC_SCRATCH_BYTES (MF_NOALLOC_MAX_ROWS * 12u + 16u)

MF_API mf_status mf_head_restricted_csr_f16_noalloc(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    uint64_t rows, uint64_t hidden_size, uint64_t vocab, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MF_HEAD_H */
