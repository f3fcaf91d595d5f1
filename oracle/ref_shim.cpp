// C-ABI shim over the reference's own CPU code — TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/Makefile together with the reference's unmodified
// sources (src/cpu/operators.cpp, src/core/shape.cpp, src/grammar/*.cpp)
// into oracle/_ref/libmfref.so.  Tests use it to pin oracle/oracle.c bit for
// bit against the reference, and bench.py's reference arm times
// mfref_full_logits_masked_head_csr on the host cores.  Nothing in the
// product links or loads it.
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <thread>
#include <vector>

#include "marketforge/core/shape.hpp"
#include "marketforge/core/tensor_view.hpp"
#include "marketforge/cpu/operators.hpp"
#include "marketforge/grammar/smollm2_market_actions.hpp"

namespace {

using marketforge::ConstTensorView;
using marketforge::DType;
using marketforge::MemoryKind;
using marketforge::TensorView;

marketforge::Shape shape2(std::uint64_t a, std::uint64_t b) {
  const std::uint64_t e[2] = {a, b};
  return marketforge::make_shape(std::span<const std::uint64_t>(e, 2)).value();
}
marketforge::Shape shape1(std::uint64_t a) {
  const std::uint64_t e[1] = {a};
  return marketforge::make_shape(std::span<const std::uint64_t>(e, 1)).value();
}

constexpr std::uint32_t kInvalid = UINT32_MAX;

// Masked argmax over one row of logits with the restricted head's rules
// (include/marketforge/cuda/greedy.hpp:35-42).  Written here, not taken from
// the reference: the reference's CPU model only does the full argmax.
void masked_pick(const float* logits, const std::int32_t* ids, std::int32_t n,
                 std::uint64_t vocab, std::uint32_t* out_id, float* out_best) {
  bool invalid = n <= 0;
  for (std::int32_t k = 0; k < n && !invalid; ++k)
    if (ids[k] < 0 || static_cast<std::uint64_t>(ids[k]) >= vocab) invalid = true;
  std::uint32_t best_id = kInvalid, fallback = kInvalid;
  float best = -std::numeric_limits<float>::infinity();
  if (!invalid) {
    for (std::int32_t k = 0; k < n; ++k) {
      const auto t = static_cast<std::uint32_t>(ids[k]);
      fallback = t < fallback ? t : fallback;
      const float v = logits[t];
      if (v > best || (v == best && t < best_id)) {
        best = v;
        best_id = t;
      }
    }
  }
  *out_id = invalid ? kInvalid : (best_id != kInvalid ? best_id : fallback);
  if (out_best) *out_best = (invalid || best_id == kInvalid) ? NAN : best;
}

} // namespace

extern "C" {

// marketforge::rms_norm_f32 (src/cpu/operators.cpp:489).  Returns the
// reference's ErrorCode (0 = ok).
int mfref_rms_norm_f32(const float* x, const float* weight, std::uint64_t rows,
                       std::uint64_t hidden, float eps, float* out) {
  const auto s = marketforge::rms_norm_f32(
      ConstTensorView{x, shape2(rows, hidden), DType::f32, MemoryKind::host},
      ConstTensorView{weight, shape1(hidden), DType::f32, MemoryKind::host}, eps,
      TensorView{out, shape2(rows, hidden), DType::f32, MemoryKind::host});
  return static_cast<int>(s.code);
}

// marketforge::linear_f32 (src/cpu/operators.cpp:539).
int mfref_linear_f32(const float* x, const float* w, std::uint64_t rows,
                     std::uint64_t in_width, std::uint64_t out_width, float* out) {
  const auto s = marketforge::linear_f32(
      ConstTensorView{x, shape2(rows, in_width), DType::f32, MemoryKind::host},
      ConstTensorView{w, shape2(out_width, in_width), DType::f32, MemoryKind::host},
      TensorView{out, shape2(rows, out_width), DType::f32, MemoryKind::host});
  return static_cast<int>(s.code);
}

// The reference CPU path for a ragged batch: per row, linear_f32 over every
// vocab row of the FP32 embedding, then the masked argmax over the row's CSR
// candidates.  With at least as many rows as threads, rows are split over
// `threads` std::threads; with fewer rows, each row's vocabulary is split
// into `threads` slices, each a linear_f32 call on its slice of the
// embedding (the same per-logit arithmetic).
int mfref_full_logits_masked_head_csr(const float* hidden, const float* embedding_f32,
                                      const std::int32_t* offsets, const std::int32_t* ids,
                                      std::uint64_t rows, std::uint64_t hidden_size,
                                      std::uint64_t vocab, std::uint32_t* out_ids,
                                      float* out_best, int threads) {
  if (threads < 1) threads = 1;
  std::vector<int> codes(static_cast<std::size_t>(threads), 0);
  if (rows < static_cast<std::uint64_t>(threads)) {
    std::vector<float> logits(vocab);
    for (std::uint64_t r = 0; r < rows; ++r) {
      auto slice = [&](int t) {
        const std::uint64_t v0 = vocab * t / threads, v1 = vocab * (t + 1) / threads;
        if (v1 > v0) {
          const int code = mfref_linear_f32(hidden + r * hidden_size,
                                            embedding_f32 + v0 * hidden_size, 1, hidden_size,
                                            v1 - v0, logits.data() + v0);
          if (code != 0) codes[t] = code;
        }
      };
      std::vector<std::thread> pool;
      for (int t = 1; t < threads; ++t) pool.emplace_back(slice, t);
      slice(0);
      for (auto& th : pool) th.join();
      for (int c : codes)
        if (c != 0) return c;
      masked_pick(logits.data(), ids + offsets[r], offsets[r + 1] - offsets[r], vocab,
                  out_ids + r, out_best ? out_best + r : nullptr);
    }
    return 0;
  }
  auto work = [&](int t) {
    std::vector<float> logits(vocab);
    const std::uint64_t b = rows * t / threads, e = rows * (t + 1) / threads;
    for (std::uint64_t r = b; r < e; ++r) {
      const int code = mfref_linear_f32(hidden + r * hidden_size, embedding_f32, 1,
                                        hidden_size, vocab, logits.data());
      if (code != 0) {
        codes[t] = code;
        return;
      }
      masked_pick(logits.data(), ids + offsets[r], offsets[r + 1] - offsets[r], vocab,
                  out_ids + r, out_best ? out_best + r : nullptr);
    }
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(work, t);
  work(0);
  for (auto& th : pool) th.join();
  for (int c : codes)
    if (c != 0) return c;
  return 0;
}

} // extern "C"

namespace {

// A fixed set of worker threads reused across calls (the benchmark's
// reference arm calls once per step; spawning threads per call would be
// timed with the work).  run(f) executes f(0..n-1) with f(0) on the caller.
class Pool {
 public:
  void ensure(int n) {
    if (n == size_) return;
    stop();
    size_ = n;
    const std::uint64_t now = gen_;  // new workers wait for the next job, not a past one
    for (int t = 1; t < n; ++t) workers_.emplace_back([this, t, now] { loop(t, now); });
  }
  void run(const std::function<void(int)>& f) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      job_ = &f;
      pending_ = size_ - 1;
      ++gen_;
    }
    cv_.notify_all();
    f(0);
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [this] { return pending_ == 0; });
    job_ = nullptr;
  }
  ~Pool() { stop(); }

 private:
  void loop(int t, std::uint64_t seen) {
    for (;;) {
      const std::function<void(int)>* f;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
        if (quit_) return;
        seen = gen_;
        f = job_;
      }
      (*f)(t);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_.notify_one();
    }
  }
  void stop() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
    workers_.clear();
    quit_ = false;
    size_ = 1;
  }
  std::mutex mu_;
  std::condition_variable cv_, done_;
  std::vector<std::thread> workers_;
  const std::function<void(int)>* job_ = nullptr;
  std::uint64_t gen_ = 0;
  int pending_ = 0, size_ = 1;
  bool quit_ = false;
};

Pool& pool() {
  static Pool p;
  return p;
}

} // namespace

extern "C" {

// The reference CPU path for a ragged batch with sequences partitioned over
// `threads` host threads of a reused pool: each thread takes a contiguous
// range of rows and, per row, runs linear_f32 over every vocab row of the
// FP32 embedding, then the masked argmax over the row's CSR candidates.
int mfref_head_csr_by_sequence(const float* hidden, const float* embedding_f32,
                               const std::int32_t* offsets, const std::int32_t* ids,
                               std::uint64_t rows, std::uint64_t hidden_size,
                               std::uint64_t vocab, std::uint32_t* out_ids, float* out_best,
                               int threads) {
  if (threads < 1) threads = 1;
  pool().ensure(threads);
  std::vector<int> codes(static_cast<std::size_t>(threads), 0);
  const std::function<void(int)> work = [&](int t) {
    thread_local std::vector<float> logits;
    logits.resize(vocab);
    const std::uint64_t b = rows * t / threads, e = rows * (t + 1) / threads;
    for (std::uint64_t r = b; r < e; ++r) {
      const int code = mfref_linear_f32(hidden + r * hidden_size, embedding_f32, 1, hidden_size,
                                        vocab, logits.data());
      if (code != 0) {
        codes[t] = code;
        return;
      }
      masked_pick(logits.data(), ids + offsets[r], offsets[r + 1] - offsets[r], vocab,
                  out_ids + r, out_best ? out_best + r : nullptr);
    }
  };
  pool().run(work);
  for (int c : codes)
    if (c != 0) return c;
  return 0;
}

// Dumps the SmolLM2 market-action DFA (SmolLm2MarketActionCatalog::create,
// src/grammar/smollm2_market_actions.cpp:42) as CSR: state s has arcs
// [offsets[s], offsets[s+1]) with tokens[] and next[] in the order
// ActionDfa::allowed returns them (sorted by token).  terminal[s] = 1 when
// ActionDfa::terminal(s).  Call with null arrays to get the counts.
int mfref_market_dfa(std::uint32_t* num_states, std::uint32_t* num_arcs,
                     std::int32_t* offsets, std::uint32_t* tokens,
                     std::uint32_t* next, std::uint8_t* terminal) {
  auto catalog = marketforge::SmolLm2MarketActionCatalog::create();
  if (!catalog) return static_cast<int>(catalog.status().code);
  const auto& dfa = catalog.value().dfa();
  *num_states = static_cast<std::uint32_t>(dfa.state_count());
  *num_arcs = static_cast<std::uint32_t>(dfa.arc_count());
  if (!offsets) return 0;
  std::int32_t at = 0;
  for (std::uint32_t s = 0; s < *num_states; ++s) {
    offsets[s] = at;
    const auto arcs = dfa.allowed(marketforge::GrammarState{s});
    if (!arcs) return static_cast<int>(arcs.status().code);
    for (const auto& arc : arcs.value()) {
      tokens[at] = arc.token;
      next[at] = arc.next.value;
      ++at;
    }
    terminal[s] = dfa.terminal(marketforge::GrammarState{s}) ? 1 : 0;
  }
  offsets[*num_states] = at;
  return 0;
}

// ActionDfa::advance (src/grammar/action_dfa.cpp:123-144) on the market DFA:
// returns the next state, or UINT32_MAX when the token is not allowed.
std::uint32_t mfref_market_dfa_advance(std::uint32_t state, std::uint32_t token) {
  static auto catalog = marketforge::SmolLm2MarketActionCatalog::create();
  if (!catalog) return kInvalid;
  const auto r = catalog.value().dfa().advance(marketforge::GrammarState{state}, token);
  return r ? r.value().value : kInvalid;
}

} // extern "C"
