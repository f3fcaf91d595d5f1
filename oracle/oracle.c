/*
 * CPU oracle for the DFA-restricted output head — TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference's CPU algorithm for the
 * hot path so that tests, the smoke check and the bench's CPU-baseline leg
 * can check the CUDA kernels against it.  The product (market_sim_b200) never
 * links, loads or calls it.
 *
 * Parity is pinned two ways (see tests/test_oracle_pin.py):
 *   - against the reference's own known-answer tests, restated as golden
 *     fixtures under tests/golden/ (tests/cuda/cuda_tests.cu:508-565,
 *     :567-697, :699-800, :1341-1404 and the pr4 greedy logits fixture);
 *   - against the reference's own compiled CPU operators (oracle/_ref, built
 *     from src/cpu/operators.cpp by oracle/Makefile), bit for bit.
 *
 * Arithmetic rules that make the comparison exact:
 *   - every dot product is the sequential FP32 loop `sum += x[i] * w[i]`
 *     with no FMA contraction (compiled with -ffp-contract=off), exactly as
 *     linear_f32 in src/cpu/operators.cpp:586-593;
 *   - fp16 inputs are widened exactly to FP32 before use.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_INVALID 0xFFFFFFFFu

/* ---- fp16 <-> fp32 widening (exact) ------------------------------------ */

/* IEEE binary16 -> binary32, exact for every input (normals, subnormals,
 * zeros, infinities, NaNs keep their payload's top bits). */
float orc_half_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {
    /* subnormal: value = man * 2^-24; normalise */
    int e = -1;
    do {
      man <<= 1;
      ++e;
    } while ((man & 0x400u) == 0);
    man &= 0x3FFu;
    bits = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

void orc_half_to_float_array(const uint16_t* in, float* out, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) out[i] = orc_half_to_float(in[i]);
}

/* ---- reference operators ------------------------------------------------ */

/* src/cpu/operators.cpp:489-537 (rms_norm_f32): sequential sum of squares,
 * inverse_rms = 1 / sqrt(mean + eps), out = x * inverse_rms * weight. */
void orc_rms_norm_f32(const float* x, const float* weight, uint64_t rows,
                      uint64_t hidden, float eps, float* out) {
  for (uint64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * hidden;
    float sum_squares = 0.0f;
    for (uint64_t c = 0; c < hidden; ++c) sum_squares += xr[c] * xr[c];
    const float inv = 1.0f / sqrtf(sum_squares / (float)hidden + eps);
    for (uint64_t c = 0; c < hidden; ++c) out[r * hidden + c] = xr[c] * inv * weight[c];
  }
}

/* One output of linear_f32 (src/cpu/operators.cpp:586-593). */
static float dot_seq(const float* x, const float* w, uint64_t n) {
  float sum = 0.0f;
  for (uint64_t i = 0; i < n; ++i) sum += x[i] * w[i];
  return sum;
}

/* One dot product where the weight row is fp16 storage widened to FP32. */
static float dot_seq_h(const float* x, const uint16_t* w, uint64_t n) {
  float sum = 0.0f;
  for (uint64_t i = 0; i < n; ++i) sum += x[i] * orc_half_to_float(w[i]);
  return sum;
}

/* src/cpu/operators.cpp:539-597 (linear_f32): out[r, o] = sum_i x[r,i] W[o,i]. */
void orc_linear_f32(const float* x, const float* w, uint64_t rows, uint64_t in_width,
                    uint64_t out_width, float* out) {
  for (uint64_t r = 0; r < rows; ++r)
    for (uint64_t o = 0; o < out_width; ++o)
      out[r * out_width + o] = dot_seq(x + r * in_width, w + o * in_width, in_width);
}

/* ---- selection rules ---------------------------------------------------- */

/* The reference's comparison (src/cuda/greedy.cu:134-212, contract in
 * include/marketforge/cuda/greedy.hpp:35-42): a candidate replaces the best
 * when its score is greater, or equal with a lower id.  NaN compares false
 * both ways, so it never wins.  Runner-up = best score among the other
 * candidates, NaN-free (the margin used by the acceptance rule). */
typedef struct {
  uint32_t best_id;
  float best;
  float runner_up;
  uint32_t fallback; /* lowest candidate id */
} orc_pick;

static void pick_init(orc_pick* p) {
  p->best_id = ORC_INVALID;
  p->best = -INFINITY;
  p->runner_up = -INFINITY;
  p->fallback = ORC_INVALID;
}

static void pick_offer(orc_pick* p, uint32_t id, float v) {
  if (id < p->fallback) p->fallback = id;
  if (v > p->best || (v == p->best && id < p->best_id)) {
    if (p->best_id != ORC_INVALID && p->best > p->runner_up) p->runner_up = p->best;
    p->best = v;
    p->best_id = id;
  } else if (v > p->runner_up) {
    p->runner_up = v;
  }
}

/* Final id: best non-NaN candidate, else (all NaN) the lowest candidate id. */
static uint32_t pick_result(const orc_pick* p) {
  return p->best_id != ORC_INVALID ? p->best_id : p->fallback;
}

/* ---- the restricted head (CSR form) -------------------------------------
 *
 * For row r the candidate set is ids[offsets[r] .. offsets[r+1]).  The score
 * of candidate t is the linear_f32 logit of t (sequential FP32 dot of the
 * widened hidden row with the widened embedding row t).  The selected id
 * follows the rules above.  Rows with zero candidates or any candidate id
 * >= vocab produce ORC_INVALID (src/cuda/greedy.cu:149-167,207-210).
 *
 * Outputs (any may be NULL): out_ids[r], out_best[r] (score of the selected
 * id; NaN when every candidate is NaN), out_runner_up[r]. */
typedef struct {
  const float* hidden;
  const uint16_t* embedding;
  const int32_t* offsets;
  const int32_t* ids;
  uint64_t hidden_size, vocab;
  uint32_t* out_ids;
  float* out_best;
  float* out_runner_up;
  uint64_t row_begin, row_end;
} head_job;

static void head_rows(const head_job* j) {
  for (uint64_t r = j->row_begin; r < j->row_end; ++r) {
    const int32_t b = j->offsets[r], e = j->offsets[r + 1];
    orc_pick p;
    pick_init(&p);
    int invalid = e <= b;
    for (int32_t k = b; k < e && !invalid; ++k)
      if (j->ids[k] < 0 || (uint64_t)j->ids[k] >= j->vocab) invalid = 1;
    if (!invalid) {
      const float* h = j->hidden + r * j->hidden_size;
      for (int32_t k = b; k < e; ++k) {
        const uint32_t t = (uint32_t)j->ids[k];
        pick_offer(&p, t, dot_seq_h(h, j->embedding + (uint64_t)t * j->hidden_size, j->hidden_size));
      }
    }
    const uint32_t id = invalid ? ORC_INVALID : pick_result(&p);
    if (j->out_ids) j->out_ids[r] = id;
    if (j->out_best) j->out_best[r] = (invalid || p.best_id == ORC_INVALID) ? NAN : p.best;
    if (j->out_runner_up) j->out_runner_up[r] = p.runner_up;
  }
}

static void* head_thread(void* arg) {
  head_rows((const head_job*)arg);
  return NULL;
}

/* Multi-threaded over rows (rows are independent; each row's arithmetic is
 * identical to the single-threaded loop). threads <= 1 runs inline. */
void orc_restricted_head_csr(const float* hidden, const uint16_t* embedding,
                             const int32_t* offsets, const int32_t* ids, uint64_t rows,
                             uint64_t hidden_size, uint64_t vocab, uint32_t* out_ids,
                             float* out_best, float* out_runner_up, int threads) {
  if (threads < 1) threads = 1;
  if ((uint64_t)threads > rows) threads = (int)(rows ? rows : 1);
  head_job* jobs = (head_job*)calloc((size_t)threads, sizeof(head_job));
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  for (int t = 0; t < threads; ++t) {
    head_job j = {hidden, embedding, offsets, ids, hidden_size, vocab,
                  out_ids, out_best, out_runner_up,
                  rows * (uint64_t)t / (uint64_t)threads,
                  rows * (uint64_t)(t + 1) / (uint64_t)threads};
    jobs[t] = j;
  }
  if (threads == 1) {
    head_rows(&jobs[0]);
  } else {
    for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, head_thread, &jobs[t]);
    for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
  }
  free(jobs);
  free(tids);
}

/* The literal reference path for one batch: full logits over every vocab row
 * (linear_f32), then the masked argmax over the row's candidates.  Used as
 * the timed CPU baseline; the selected ids equal orc_restricted_head_csr's
 * because each logit is an independent sequential dot.  `logits_scratch`
 * holds threads * vocab floats. */
typedef struct {
  head_job base;
  float* logits;
} full_job;

static void* full_thread(void* arg) {
  full_job* f = (full_job*)arg;
  const head_job* j = &f->base;
  for (uint64_t r = j->row_begin; r < j->row_end; ++r) {
    const float* h = j->hidden + r * j->hidden_size;
    for (uint64_t t = 0; t < j->vocab; ++t)
      f->logits[t] = dot_seq_h(h, j->embedding + t * j->hidden_size, j->hidden_size);
    const int32_t b = j->offsets[r], e = j->offsets[r + 1];
    orc_pick p;
    pick_init(&p);
    int invalid = e <= b;
    for (int32_t k = b; k < e && !invalid; ++k)
      if (j->ids[k] < 0 || (uint64_t)j->ids[k] >= j->vocab) invalid = 1;
    if (!invalid)
      for (int32_t k = b; k < e; ++k) pick_offer(&p, (uint32_t)j->ids[k], f->logits[j->ids[k]]);
    if (j->out_ids) j->out_ids[r] = invalid ? ORC_INVALID : pick_result(&p);
    if (j->out_best) j->out_best[r] = (invalid || p.best_id == ORC_INVALID) ? NAN : p.best;
    if (j->out_runner_up) j->out_runner_up[r] = p.runner_up;
  }
  return NULL;
}

void orc_full_logits_masked_head_csr(const float* hidden, const uint16_t* embedding,
                                     const int32_t* offsets, const int32_t* ids,
                                     uint64_t rows, uint64_t hidden_size, uint64_t vocab,
                                     uint32_t* out_ids, float* out_best, int threads) {
  if (threads < 1) threads = 1;
  if ((uint64_t)threads > rows) threads = (int)(rows ? rows : 1);
  full_job* jobs = (full_job*)calloc((size_t)threads, sizeof(full_job));
  pthread_t* tids = (pthread_t*)calloc((size_t)threads, sizeof(pthread_t));
  float* logits = (float*)malloc((size_t)threads * vocab * sizeof(float));
  for (int t = 0; t < threads; ++t) {
    head_job j = {hidden, embedding, offsets, ids, hidden_size, vocab,
                  out_ids, out_best, NULL,
                  rows * (uint64_t)t / (uint64_t)threads,
                  rows * (uint64_t)(t + 1) / (uint64_t)threads};
    jobs[t].base = j;
    jobs[t].logits = logits + (size_t)t * vocab;
  }
  if (threads == 1) {
    full_thread(&jobs[0]);
  } else {
    for (int t = 0; t < threads; ++t) pthread_create(&tids[t], NULL, full_thread, &jobs[t]);
    for (int t = 0; t < threads; ++t) pthread_join(tids[t], NULL);
  }
  free(logits);
  free(jobs);
  free(tids);
}

/* ---- selection over materialised fp16 logits ---------------------------- */

/* src/cuda/greedy.cu:21-59 (greedy_kernel): argmax over all columns with the
 * lowest-id tie rule; a row whose every logit is NaN selects token 0. */
void orc_greedy_select_f16(const uint16_t* logits, uint64_t rows, uint64_t vocab,
                           uint32_t* out) {
  for (uint64_t r = 0; r < rows; ++r) {
    orc_pick p;
    pick_init(&p);
    for (uint64_t t = 0; t < vocab; ++t)
      pick_offer(&p, (uint32_t)t, orc_half_to_float(logits[r * vocab + t]));
    out[r] = p.best_id == ORC_INVALID ? 0u : p.best_id;
  }
}

/* src/cuda/greedy.cu:61-131 (restricted_greedy_kernel): masked argmax over a
 * padded [rows, max_allowed] candidate table with per-row counts.  count 0,
 * count > max_allowed or any candidate >= vocab -> ORC_INVALID; all NaN ->
 * lowest candidate id. */
void orc_restricted_greedy_select_f16(const uint16_t* logits, const uint32_t* allowed,
                                      const uint32_t* counts, uint64_t rows, uint64_t vocab,
                                      uint64_t max_allowed, uint32_t* out) {
  for (uint64_t r = 0; r < rows; ++r) {
    const uint32_t n = counts[r];
    int invalid = n == 0 || n > max_allowed;
    for (uint32_t k = 0; k < n && !invalid; ++k)
      if (allowed[r * max_allowed + k] >= vocab) invalid = 1;
    orc_pick p;
    pick_init(&p);
    if (!invalid)
      for (uint32_t k = 0; k < n; ++k) {
        const uint32_t t = allowed[r * max_allowed + k];
        pick_offer(&p, t, orc_half_to_float(logits[r * vocab + t]));
      }
    out[r] = invalid ? ORC_INVALID : pick_result(&p);
  }
}

/* The padded-table restricted head (restricted_output_head_f16's contract,
 * include/marketforge/cuda/greedy.hpp:35-49): same rules as the CSR form,
 * with count > max_allowed also invalid. */
void orc_restricted_head_padded(const float* hidden, const uint16_t* embedding,
                                const uint32_t* allowed, const uint32_t* counts,
                                uint64_t rows, uint64_t hidden_size, uint64_t vocab,
                                uint64_t max_allowed, uint32_t* out_ids, float* out_best) {
  for (uint64_t r = 0; r < rows; ++r) {
    const uint32_t n = counts[r];
    int invalid = n == 0 || n > max_allowed;
    for (uint32_t k = 0; k < n && !invalid; ++k)
      if (allowed[r * max_allowed + k] >= vocab) invalid = 1;
    orc_pick p;
    pick_init(&p);
    if (!invalid)
      for (uint32_t k = 0; k < n; ++k) {
        const uint32_t t = allowed[r * max_allowed + k];
        pick_offer(&p, t, dot_seq_h(hidden + r * hidden_size,
                                    embedding + (uint64_t)t * hidden_size, hidden_size));
      }
    out_ids[r] = invalid ? ORC_INVALID : pick_result(&p);
    if (out_best) out_best[r] = (invalid || p.best_id == ORC_INVALID) ? NAN : p.best;
  }
}

/* ---- dense full-vocab head ----------------------------------------------
 *
 * Full logits over vocab rows [vocab_begin, vocab_end) (linear_f32 order),
 * argmax with the lowest-id tie rule; all-NaN rows select vocab_begin
 * (greedy_select_f16's "token 0" rule applied to the slice).  Also returns
 * the best score and runner-up score for the acceptance margin. */
void orc_dense_head(const float* hidden, const uint16_t* embedding, uint64_t rows,
                    uint64_t hidden_size, uint64_t vocab_begin, uint64_t vocab_end,
                    uint32_t* out_ids, float* out_best, float* out_runner_up) {
  for (uint64_t r = 0; r < rows; ++r) {
    orc_pick p;
    pick_init(&p);
    for (uint64_t t = vocab_begin; t < vocab_end; ++t)
      pick_offer(&p, (uint32_t)t,
                 dot_seq_h(hidden + r * hidden_size, embedding + t * hidden_size, hidden_size));
    out_ids[r] = p.best_id == ORC_INVALID ? (uint32_t)vocab_begin : p.best_id;
    if (out_best) out_best[r] = p.best_id == ORC_INVALID ? NAN : p.best;
    if (out_runner_up) out_runner_up[r] = p.runner_up;
  }
}

/* ---- synthetic token DFA and multi-step constrained decode --------------
 *
 * The DFA is CSR: state s allows ids[offsets[s] .. offsets[s+1]) (the flat
 * form of TokenDfa's StateRecord{first_arc, arc_count} + arcs,
 * include/marketforge/grammar/token_dfa.hpp:54-58).  The synthetic grammar's
 * transition is next = splitmix64(((uint64)state << 32) | token) mod states.
 * Multi-step decode: for each step and sequence, pick with the restricted
 * head from the sequence's state's allowed set, then advance. */
uint64_t orc_splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

uint32_t orc_dfa_next(uint32_t state, uint32_t token, uint32_t num_states) {
  return (uint32_t)(orc_splitmix64(((uint64_t)state << 32) | token) % num_states);
}

/* TokenDfa::advance (src/grammar/token_dfa.cpp:111-128): lower_bound of the
 * token in the state's sorted arcs; returns the arc index or -1. */
static int64_t arc_of(const int32_t* dfa_offsets, const int32_t* dfa_ids, uint32_t state,
                      uint32_t token) {
  int64_t lo = dfa_offsets[state], hi = dfa_offsets[state + 1];
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo) / 2;
    if ((uint32_t)dfa_ids[mid] < token) lo = mid + 1; else hi = mid;
  }
  return (lo < dfa_offsets[state + 1] && (uint32_t)dfa_ids[lo] == token) ? lo : -1;
}

/* hidden: [steps, batch, hidden_size] FP32 (widened fp16); init_states[batch];
 * out_tokens: [steps, batch]; out_states: [steps + 1, batch].  arc_next may be
 * NULL (synthetic hash transition) or the DFA's per-arc next-state table
 * (TokenDfa::advance).  States out of range or without arcs give
 * ORC_INVALID and keep their state. */
void orc_dfa_decode(const float* hidden, const uint16_t* embedding,
                    const int32_t* dfa_offsets, const int32_t* dfa_ids, const uint32_t* arc_next,
                    uint32_t num_states, const uint32_t* init_states, uint64_t steps,
                    uint64_t batch, uint64_t hidden_size, uint64_t vocab, uint32_t* out_tokens,
                    uint32_t* out_states) {
  uint32_t* state = (uint32_t*)malloc(batch * sizeof(uint32_t));
  memcpy(state, init_states, batch * sizeof(uint32_t));
  memcpy(out_states, state, batch * sizeof(uint32_t));
  for (uint64_t s = 0; s < steps; ++s) {
    for (uint64_t b = 0; b < batch; ++b) {
      const uint32_t st = state[b];
      uint32_t tok = ORC_INVALID;
      if (st < num_states && dfa_offsets[st + 1] > dfa_offsets[st]) {
        int32_t off[2] = {dfa_offsets[st], dfa_offsets[st + 1]};
        int32_t rel[2] = {0, off[1] - off[0]};
        head_job j = {hidden + (s * batch + b) * hidden_size, embedding, rel, dfa_ids + off[0],
                      hidden_size, vocab, &tok, NULL, NULL, 0, 1};
        head_rows(&j);
      }
      out_tokens[s * batch + b] = tok;
      if (tok != ORC_INVALID) {
        if (arc_next) {
          const int64_t a = arc_of(dfa_offsets, dfa_ids, st, tok);
          if (a >= 0) state[b] = arc_next[a];
        } else {
          state[b] = orc_dfa_next(st, tok, num_states);
        }
      }
    }
    memcpy(out_states + (s + 1) * batch, state, batch * sizeof(uint32_t));
  }
  free(state);
}
