// Ragged (CSR) restricted output head and the device-resident DFA step.
//
// Reference behaviour: restricted_output_head_kernel, src/cuda/greedy.cu:133-212
// (one thread block per row, one thread per candidate walking the 576-wide
// row 2 bytes at a time).  Here the candidates of the whole batch are laid
// out flat (CSR) and split evenly over every 8-lane group on the GPU, so a
// 4096-candidate row is shared by hundreds of groups while a 1-candidate row
// costs one group-iteration:
//
//   * a group of 8 lanes reads one embedding row per iteration as 9 x 16 B
//     coalesced loads per lane (1152 B per row), two rows in flight;
//   * the hidden row sits in registers as fp16 (36 x u32 per lane) and the
//     dot product uses sm_100's f16 x f16 -> f32 FMA, then a 3-step shuffle;
//   * each group keeps a running packed (score, id) key per row; a row owned
//     by one group is finalised straight from registers, a row shared by
//     several groups merges with atomicMax on a 64-bit key in the workspace
//     and the group that completes the row's candidate count finalises it
//     (per-row arrival counter).  Max is order-independent, so results are
//     deterministic.
//
// Workspace layout (zero between calls; every call returns it to zero):
//   keys  u64[rows] | count u32[rows] | control u32[4] (done, anomaly, -, -)
#include <cuda_runtime.h>

#include <initializer_list>
#include <utility>
#include <mutex>

#include "common.cuh"

namespace mfb {

enum class RowMode { kCsr, kDfa };

struct RaggedParams {
  const __half* hidden;
  const __half* embedding;
  // CSR mode: offsets[rows+1] and ids[total].
  const int32_t* offsets;
  const int32_t* ids;
  // CSR mode, vocabularies of at most 65,536 ids: the candidates as u16
  // instead of `ids` (half the bytes to move from the host); null: `ids`
  const uint16_t* ids16;
  int64_t total;
  // DFA mode: states_in[rows] index state_offsets[num_states+1] into
  // arc_tokens / arc_next[num_arcs].
  const int32_t* state_offsets;
  const uint32_t* arc_next;
  const uint32_t* states_in;
  uint32_t* states_out;
  uint32_t num_states;
  // DFA mode with vocab <= 65,536 and num_states < 65,535: a key's id field
  // packs (token << 16 | next state) instead of the arc's position, so the
  // row's finaliser needs no table loads (arcs are sorted by token, so the
  // lowest token is the lowest position: the selection order is the same).
  uint32_t dfa_packed;
  // Multi-step decode with packed keys (mf_dfa_decode_f16): a step's rows
  // merge into dfa_keys_out by atomicMax alone (no arrival counters, no
  // finaliser); the next step's prologue decodes them into the previous
  // step's token / score / state rows.  Three key buffers rotate: step s
  // writes K[s % 3], reads K[(s - 1) % 3] and clears K[(s + 1) % 3], which
  // step s - 1's prologue has finished reading.  Null: the per-row merge.
  unsigned long long* dfa_keys_out;
  const unsigned long long* dfa_keys_in;  // the previous step's keys, or null (first step)
  unsigned long long* dfa_keys_clear;
  const uint32_t* states_prev;   // the previous step's input states
  uint32_t* states_in_w;         // this step's input state row (written from the keys)
  uint32_t* prev_out_ids;        // the previous step's token row
  float* prev_out_scores;        // the previous step's score row, or null
  int64_t num_arcs;
  // outputs
  uint32_t* out_ids;
  float* out_scores;
  // workspace
  unsigned long long* keys;
  uint32_t* counts;
  uint32_t* control;
  uint32_t rows;
  uint32_t hidden_size;
  uint32_t vocab;
  // Fused final RMSNorm (optional): when gamma is set, `hidden` holds the
  // un-normalised rows and each is normalised in registers first.
  const __half* gamma;
  float eps;
};

constexpr int kThreads = 256;
constexpr int kGroupsPerBlock = kThreads / 8;
constexpr int kMaxDfaBatch = 8192;
// CSR batches of up to this many rows are validated by every block on its
// own (each thread reads at most 16 offsets): a block that finds the offsets
// malformed gives its share of the rows the sentinel and computes nothing,
// so no block needs to hear from the others and the kernel ends without a
// grid-wide arrival counter.  Larger batches keep the counter: the last
// block out checks a flag the others raised.
constexpr uint32_t kLocalCheckRows = 16 * kThreads;

// Row-start table for one row mode.  CSR reads global offsets; DFA mode
// builds the prefix sum of the allowed-set sizes in shared memory.
template <RowMode M>
struct Rows;

template <>
struct Rows<RowMode::kCsr> {
  const int32_t* start;  // global, rows + 1 entries
  __device__ __forceinline__ int64_t at(uint32_t r) const { return start[r]; }
};

template <>
struct Rows<RowMode::kDfa> {
  const int32_t* start;     // shared, rows + 1 entries
  const int32_t* arc_base;  // shared, rows entries: first arc of each row's state
  __device__ __forceinline__ int64_t at(uint32_t r) const { return start[r]; }
};

// Largest r in [0, rows) with at(r) <= c (rows assumed non-decreasing);
// 8-ary search shared by the 8 lanes of a group.
template <RowMode M>
__device__ uint32_t find_row(const Rows<M>& rows_tab, uint32_t rows, int64_t c, int sub,
                             unsigned gmask) {
  uint32_t lo = 0, hi = rows;  // answer in [lo, hi)
  while (hi - lo > 1) {
    const uint32_t span = hi - lo;
    const uint32_t step = (span + 7) / 8;
    const uint32_t probe = lo + (uint32_t)sub * step;
    const bool ok = probe < hi && rows_tab.at(probe) <= c;
    const unsigned ballot = __ballot_sync(gmask, ok) & gmask;
    // lanes are ordered by probe; the last lane with ok gives the new lo
    const int last = 31 - __clz(ballot);
    const int lane_base = (threadIdx.x & 31) & ~7;
    const uint32_t new_lo = lo + (uint32_t)(last >= 0 ? last - lane_base : 0) * step;
    const uint32_t new_hi = min(hi, new_lo + step);
    lo = new_lo;
    hi = new_hi;
  }
  return lo;
}

// Writes the final result of row r from its merged key.
template <RowMode M>
__device__ void finalize_row(const RaggedParams& p, const Rows<M>& rows_tab, uint32_t r,
                             unsigned long long key) {
  if constexpr (M == RowMode::kCsr) {
    const bool ok = key_is_result(key);
    p.out_ids[r] = ok ? key_id(key) : kInvalid;
    if (p.out_scores) p.out_scores[r] = ok ? key_score(key) : __uint_as_float(0x7FC00000u);
  } else {
    if (p.dfa_packed && key_is_result(key)) {
      p.out_ids[r] = key_id(key) >> 16;
      p.states_out[r] = key_id(key) & 0xFFFFu;
      if (p.out_scores) p.out_scores[r] = key_score(key);
      return;
    }
    const uint32_t st = p.states_in[r];
    if (key_is_result(key)) {
      const int64_t arc = (int64_t)rows_tab.arc_base[r] + key_id(key);
      p.out_ids[r] = (uint32_t)p.ids[arc];
      p.states_out[r] = p.arc_next[arc];
      if (p.out_scores) p.out_scores[r] = key_score(key);
    } else {
      p.out_ids[r] = kInvalid;
      p.states_out[r] = st;
      if (p.out_scores) p.out_scores[r] = __uint_as_float(0x7FC00000u);
    }
  }
}

// Load the hidden row r's 9 chunks owned by this lane (fast path).
__device__ __forceinline__ void load_hidden_fast(const __half* hidden, uint32_t r, int sub,
                                                 uint4 (&h)[kFastChunksPerLane]) {
  const uint4* row = reinterpret_cast<const uint4*>(hidden + (size_t)r * kFastHidden);
#pragma unroll
  for (int k = 0; k < kFastChunksPerLane; ++k) h[k] = ld_v4(row + sub + 8 * k);
}

// Stages hidden row r's 9 chunks owned by this lane into its shared-memory
// slot (slot[k * kThreads], k = 0..8), normalised first when gamma is set
// (what the reference's rms_norm_f16, src/cuda/rms_norm.cu:69-100, would
// store: inv = 1 / sqrt(mean(x^2) + eps) in FP32, h = fp16(x * inv * w), the
// order of src/cpu/operators.cpp:522-535).  Two passes over the slot keep at
// most one row's chunks in registers.
template <bool kNorm>
__device__ __forceinline__ void stage_hidden_fast(const __half* hidden, uint32_t r, int sub,
                                                  unsigned gmask, const __half* gamma, float eps,
                                                  uint4* slot) {
  uint4 h[kFastChunksPerLane];
  load_hidden_fast(hidden, r, sub, h);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kFastChunksPerLane; ++k) {
    slot[k * kThreads] = h[k];
    if (kNorm) {
      const uint32_t w[4] = {h[k].x, h[k].y, h[k].z, h[k].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
  }
  if (!kNorm) return;
  ss = group8_sum(ss, gmask);
  const float inv = 1.0f / sqrtf(ss / (float)kFastHidden + eps);
  const uint4* g = reinterpret_cast<const uint4*>(gamma);
#pragma unroll
  for (int k = 0; k < kFastChunksPerLane; ++k) {
    const uint4 gv = ld_v4(g + sub + 8 * k);
    const uint4 hv = slot[k * kThreads];
    uint32_t w[4] = {hv.x, hv.y, hv.z, hv.w};
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&gw[j]));
      const __half2 o = __floats2half2_rn(x.x * inv * y.x, x.y * inv * y.y);
      w[j] = *reinterpret_cast<const uint32_t*>(&o);
    }
    slot[k * kThreads] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// inv_rms of hidden row r for the generic path (1 when not normalising).
__device__ float row_inv_rms(const RaggedParams& p, uint32_t r, int sub, unsigned gmask) {
  if (p.gamma == nullptr) return 1.f;
  const __half* x = p.hidden + (size_t)r * p.hidden_size;
  float ss = 0.f;
  for (uint32_t f = sub; f < p.hidden_size; f += 8) {
    const float v = __half2float(x[f]);
    ss = fmaf(v, v, ss);
  }
  ss = group8_sum(ss, gmask);
  return 1.0f / sqrtf(ss / (float)p.hidden_size + p.eps);
}

// Dot product of hidden row r with embedding row t by one 8-lane group:
// generic path for any width (used by the small known-answer shapes).  With
// a gamma, the hidden element is normalised and rounded to fp16 first.
__device__ float group_dot_generic(const RaggedParams& p, uint32_t r, uint32_t t, float inv,
                                   int sub, unsigned gmask) {
  const uint32_t width = p.hidden_size;
  float a = 0.f;
  const __half* h = p.hidden + (size_t)r * width;
  const __half* e = p.embedding + (size_t)t * width;
  for (uint32_t f = sub; f < width; f += 8) {
    float hv = __half2float(h[f]);
    if (p.gamma != nullptr) hv = __half2float(__float2half_rn(hv * inv * __half2float(p.gamma[f])));
    a = fmaf(hv, __half2float(e[f]), a);
  }
  return group8_sum(a, gmask);
}

// Row arrival counter: a release-acquire add at GPU scope, so this group's
// earlier key merge is visible to whichever group completes the row, and the
// completing group sees every other group's merge (lighter than a full
// fence around a relaxed add).
__device__ __forceinline__ uint32_t arrive_acq_rel(uint32_t* counter, uint32_t n) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(counter), "r"(n)
               : "memory");
  return old;
}

// Per-block merge slots: the groups of a block cover one contiguous range of
// flat candidates, and each group is the first group of the block to touch at
// most one row that continues into later groups (its last row), so slot g
// (g = first toucher) holds that row's partial key and candidate count.
struct BlockSlots {
  unsigned long long* key;  // shared [kGroupsPerBlock]
  uint32_t* count;          // shared [kGroupsPerBlock]
  int64_t begin, end;       // the block's flat candidate range
  int64_t chunk;            // candidates per group
};

// CSR batches of up to kLocalCheckRows rows on more than one block: each
// block's part of a row goes to the row key by one atomicMax that nothing
// waits on, and a finishing kernel decodes every key after the whole grid (no
// arrival counter, no finaliser on the critical path of a block).  A
// one-block grid finalises its rows itself: every row then completes inside
// the block's shared-memory merge, so no global key is touched and a second
// launch would only add latency.
__device__ __forceinline__ bool csr_keys_only(const RaggedParams& p) {
  return p.rows <= kLocalCheckRows && gridDim.x > 1;
}

// Malformed offsets found by the per-block check: with the finishing kernel
// every row key stays zero and decodes to the sentinel; a one-block grid
// writes the sentinels itself.
__device__ __forceinline__ void csr_malformed(const RaggedParams& p) {
  if (csr_keys_only(p)) return;
  pdl_wait();
  for (uint32_t r = threadIdx.x; r < p.rows; r += kThreads) {
    p.out_ids[r] = kInvalid;
    if (p.out_scores) p.out_scores[r] = __uint_as_float(0x7FC00000u);
  }
}

// One flushed (row, key, n) triple: merge and finalise when complete.  A
// row split between groups first merges in the block's shared slot; only
// the group that completes the block's part of the row goes on to the
// global key / arrival counter (so a long row costs one global merge per
// block, not one per group).
template <RowMode M>
__device__ void flush_row(const RaggedParams& p, const Rows<M>& rows_tab, uint32_t r,
                          int64_t row_b, int64_t row_e, unsigned long long key, int64_t n,
                          int sub, const BlockSlots& bs) {
  if (sub != 0 || n <= 0) return;
  if constexpr (M == RowMode::kDfa) {
    if (p.dfa_keys_out != nullptr) {  // decoded by the next step's prologue
      if (key != kKeyNone) atomicMax(p.dfa_keys_out + r, key);
      return;
    }
  }
  pdl_wait();  // the workspace and outputs may still belong to the previous launch
  const int64_t row_len = row_e - row_b;
  const bool keys_only = M == RowMode::kCsr && csr_keys_only(p);
  if (n == row_len && !keys_only) {  // the group saw the whole row: no merge needed
    finalize_row<M>(p, rows_tab, r, key);
    return;
  }
  const int64_t lb = max(row_b, bs.begin), le = min(row_e, bs.end);
  const int64_t local = le - lb;
  if (n < local && lb >= bs.begin) {  // shared with other groups of this block
    const int slot = (int)((lb - bs.begin) / bs.chunk);
    atomicMax(bs.key + slot, key);
    __threadfence_block();
    const uint32_t before = atomicAdd(bs.count + slot, (uint32_t)n);
    if ((int64_t)before + n != local) return;
    __threadfence_block();
    key = atomicExch(bs.key + slot, 0ull);
    n = local;
    if (n == row_len && !keys_only) {  // the row lies inside this block
      finalize_row<M>(p, rows_tab, r, key);
      return;
    }
  }
  if (keys_only) {
    if (key != kKeyNone) atomicMax(p.keys + r, key);
    return;
  }
  if (key != kKeyNone) atomicMax(p.keys + r, key);
  const uint32_t before = arrive_acq_rel(p.counts + r, (uint32_t)n);
  if ((int64_t)before + n == row_len) {
    const unsigned long long merged = atomicExch(p.keys + r, 0ull);
    p.counts[r] = 0u;
    finalize_row<M>(p, rows_tab, r, merged);
  }
}

// Batches of up to kLocalCheckRows rows: one pass of the block over the
// offsets.  It checks them (non-decreasing, offsets[0] = 0, offsets[rows] =
// total) and counts how many rows start at or before the block's first and
// last candidate, which gives the rows [first, last] that the block's range
// [b_begin, b_end) covers without a search.  false: malformed (the whole
// block returns; every block finds the same, so no block merges a key and the
// finishing kernel gives every row the sentinel).
__device__ __forceinline__ bool csr_local_check(const RaggedParams& p, int64_t b_begin,
                                                int64_t b_end, uint32_t (*s_row_counts)[2],
                                                uint32_t& first, uint32_t& last) {
  const int64_t b0 = b_begin, b1 = b_end - 1;
  int bad = 0;
  uint32_t n0 = 0, n1 = 0;
  for (uint32_t r = threadIdx.x; r < p.rows; r += kThreads) {
    const int32_t o = __ldg(p.offsets + r);
    bad |= o > __ldg(p.offsets + r + 1);
    n0 += (int64_t)o <= b0;
    n1 += (int64_t)o <= b1;
  }
  if (threadIdx.x == 0)
    bad |= __ldg(p.offsets) != 0 || (int64_t)__ldg(p.offsets + p.rows) != p.total;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    n0 += __shfl_xor_sync(0xFFFFFFFFu, n0, o);
    n1 += __shfl_xor_sync(0xFFFFFFFFu, n1, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_row_counts[threadIdx.x >> 5][0] = n0;
    s_row_counts[threadIdx.x >> 5][1] = n1;
  }
  if (__syncthreads_or(bad)) return false;
  n0 = n1 = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    n0 += s_row_counts[w][0];
    n1 += s_row_counts[w][1];
  }
  first = n0 > 0 ? n0 - 1 : 0u;
  last = n1 > 0 ? n1 - 1 : 0u;
  return true;
}

// 16-byte asynchronous global -> shared copy (no registers on the way) and
// the wait for every such copy this thread issued.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// Rows a thread block can stage once for all its groups (the block's
// candidate range covers at most this many rows); blocks spanning more rows
// stage per group.
constexpr int kBlockRows = 16;
// Dynamic shared memory of the CSR fast path: the per-lane hidden slots and
// the block's row table.
constexpr int kCsrFastSmem = (kThreads * kFastChunksPerLane + kBlockRows * 72) * 16;

// Shared-memory row table of a block on the CSR fast path.
struct BlockRowTable {
  uint4* rows;     // [kBlockRows][72] hidden rows (normalised when fusing the norm)
  int64_t* start;  // [kBlockRows + 1] offsets of rows first .. first + n
  uint32_t first;  // first row of the block's candidate range
  int n;           // rows staged (0: the block stages per group)
};

// Warp-cooperative staging of hidden row r into dst (72 x 16 B): lane l
// owns chunks l, l + 32, l + 64 (< 72).  With the fused norm the row is
// normalised as the reference's rms_norm_f16 would store it
// (src/cuda/rms_norm.cu:69-100: inv = 1 / sqrt(mean(x^2) + eps) in FP32,
// h = fp16(x * inv * w), the order of src/cpu/operators.cpp:522-535).
template <bool kNorm>
__device__ __forceinline__ void stage_row_warp(const RaggedParams& p, uint32_t r, uint4* dst,
                                               int lane) {
  const uint4* src = reinterpret_cast<const uint4*>(p.hidden + (size_t)r * kFastHidden);
  uint4 v[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int ch = lane + 32 * j;
    v[j] = ch < 72 ? ld_v4(src + ch) : make_uint4(0, 0, 0, 0);
  }
  if (kNorm) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    const float inv = 1.0f / sqrtf(ss / (float)kFastHidden + p.eps);
    const uint4* g = reinterpret_cast<const uint4*>(p.gamma);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int ch = lane + 32 * j;
      if (ch >= 72) continue;
      const uint4 gv = ld_v4(g + ch);
      uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[q]));
        const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&gw[q]));
        const __half2 o = __floats2half2_rn(x.x * inv * y.x, x.y * inv * y.y);
        w[q] = *reinterpret_cast<const uint32_t*>(&o);
      }
      v[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
#pragma unroll
  for (int j = 0; j < 3; ++j)
    if (lane + 32 * j < 72) dst[lane + 32 * j] = v[j];
}

// The CSR fast path (576-wide rows) for a whole thread block; every thread
// calls it (it holds block barriers).  Group g of the block owns flat
// candidates [c_begin, c_end).
//   * Each group issues the embedding loads of its first two candidates at
//     once; while they are in flight the block finds the rows its range
//     covers and, when they are at most kBlockRows, stages those hidden rows
//     (normalised, when fusing the norm) and their offsets in shared memory
//     once for all groups, a warp per row.  (With the fused norm the first
//     loads wait for the staging.)
//   * Each iteration then issues the embedding loads of its (up to) two
//     candidates before settling which row they belong to, so a change of
//     row (the flush of the finished row, the next row's offsets and hidden
//     row) runs while those loads are in flight.  A second candidate that
//     turns out to open the next row is dropped and loaded again by the next
//     iteration.
//   * A block spanning more rows (many short rows) stages per group: the
//     lane's own shared-memory slot by cp.async, normalised in place.
template <bool kNorm, bool kIds16>
__device__ __forceinline__ void csr_fast_block(const RaggedParams& p,
                                               const Rows<RowMode::kCsr>& rows_tab,
                                               int64_t c_begin, int64_t c_end, int sub,
                                               unsigned gmask, uint4* slot,
                                               const BlockSlots& bs, BlockRowTable& tab,
                                               uint32_t* s_rows_found,
                                               uint32_t (*s_row_counts)[2]) {
  const uint4* emb = reinterpret_cast<const uint4*>(p.embedding);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t c = c_begin;
  uint32_t t0 = 0, t1 = 0;
  bool has1 = false, v0 = false, v1 = false;
  uint4 e0[kFastChunksPerLane], e1[kFastChunksPerLane];
  auto issue = [&]() {
    has1 = c + 1 < c_end;
    if constexpr (kIds16) {
      t0 = __ldg(p.ids16 + c);
      t1 = has1 ? __ldg(p.ids16 + c + 1) : 0u;
    } else {
      t0 = (uint32_t)__ldg(p.ids + c);
      t1 = has1 ? (uint32_t)__ldg(p.ids + c + 1) : 0u;
    }
    v0 = t0 < p.vocab;
    v1 = has1 && t1 < p.vocab;
    if (v0) {
      const uint4* row = emb + (size_t)t0 * (kFastHidden / 8) + sub;
#pragma unroll
      for (int k = 0; k < kFastChunksPerLane; ++k) e0[k] = ld_stream_v4(row + 8 * k);
    }
    if (v1) {
      const uint4* row = emb + (size_t)t1 * (kFastHidden / 8) + sub;
#pragma unroll
      for (int k = 0; k < kFastChunksPerLane; ++k) e1[k] = ld_stream_v4(row + 8 * k);
    }
  };
  // (with the fused norm, after the staging below: the rows' normalisation
  // needs the registers that two rows in flight would hold)
  if (!kNorm && c < c_end) issue();

  // ---- the block's rows: [first, last] covering [bs.begin, bs.end) ----
  // (small batches: counted by the offset check, whose loads overlap the
  // first embedding loads; the candidate indices are below total whatever
  // the offsets hold, so those loads stay in bounds)
  bool rows_known = false;
  uint32_t known_first = 0, known_last = 0;
  if (p.rows <= kLocalCheckRows) {
    if (!csr_local_check(p, bs.begin, bs.end, s_row_counts, known_first, known_last)) {
      csr_malformed(p);
      return;
    }
    rows_known = true;
  }
  if (!rows_known) {
    if (warp == 0 && lane < 16) {  // group 0: first row, group 1: last row
      const int64_t at = lane < 8 ? bs.begin : bs.end - 1;
      uint32_t r = 0;
      if (bs.begin < bs.end) r = find_row<RowMode::kCsr>(rows_tab, p.rows, at, sub, gmask);
      if (sub == 0) s_rows_found[lane >> 3] = r;
    }
    __syncthreads();
  }
  const uint32_t first = rows_known ? known_first : s_rows_found[0];
  const uint32_t last = rows_known ? known_last : s_rows_found[1];
  const int64_t span = (int64_t)last - (int64_t)first + 1;
  tab.first = first;
  tab.n = (bs.begin < bs.end && span >= 1 && span <= kBlockRows) ? (int)span : 0;
  if (tab.n > 0) {
    for (int i = warp; i < tab.n; i += kThreads / 32)
      stage_row_warp<kNorm>(p, first + (uint32_t)i, tab.rows + i * 72, lane);
    if ((int)threadIdx.x <= tab.n) tab.start[threadIdx.x] = rows_tab.at(first + threadIdx.x);
  }
  __syncthreads();
  if (kNorm && c < c_end) issue();

  // ---- the group's candidates ----
  const bool table = tab.n > 0;
  const uint4* hid = slot;  // current hidden row: chunk k at hid[k * hstride]
  const int hstride = table ? 8 : kThreads;
  uint32_t r = 0;
  int64_t row_b = 0, row_e = c_begin;  // no row yet: the first iteration finds it
  bool have_row = false, pre = true;
  unsigned long long best = kKeyNone;
  int64_t seen = 0;
  auto row_start = [&](uint32_t q) -> int64_t {
    return table ? tab.start[q - first] : rows_tab.at(q);
  };
  // Row change: flush the finished row, find the next one, point at (or
  // stage) its hidden state.  false: malformed offsets (stop).
  auto enter_row = [&]() -> bool {
    const uint32_t r_end = table ? first + (uint32_t)tab.n : p.rows;  // rows [.., r_end)
    if (have_row) {
      flush_row<RowMode::kCsr>(p, rows_tab, r, row_b, row_e, best, seen, sub, bs);
      best = kKeyNone;
      seen = 0;
      while (c >= row_e && r + 1 < r_end) {
        ++r;
        row_b = row_e;
        row_e = row_start(r + 1);
      }
    } else {
      if (table) {
        r = first;
        while (r + 1 < r_end && tab.start[r + 1 - first] <= c) ++r;
      } else {
        r = find_row<RowMode::kCsr>(rows_tab, p.rows, c, sub, gmask);
      }
      row_b = row_start(r);
      row_e = row_start(r + 1);
      have_row = true;
    }
    if (c >= row_e || c < row_b) return false;  // malformed offsets: stop
    if (table) {
      hid = tab.rows + (r - first) * 72 + sub;
      return true;
    }
    const uint4* h = reinterpret_cast<const uint4*>(p.hidden + (size_t)r * kFastHidden) + sub;
#pragma unroll
    for (int k = 0; k < kFastChunksPerLane; ++k) cp_async16(slot + k * kThreads, h + 8 * k);
    cp_async_wait_all();
    if (kNorm) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < kFastChunksPerLane; ++k) {
        const uint4 hv = slot[k * kThreads];
        const uint32_t w[4] = {hv.x, hv.y, hv.z, hv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          ss = fmaf(f.x, f.x, ss);
          ss = fmaf(f.y, f.y, ss);
        }
      }
      ss = group8_sum(ss, gmask);
      const float inv = 1.0f / sqrtf(ss / (float)kFastHidden + p.eps);
      const uint4* g = reinterpret_cast<const uint4*>(p.gamma) + sub;
#pragma unroll
      for (int k = 0; k < kFastChunksPerLane; ++k) {
        const uint4 gv = ld_v4(g + 8 * k);
        const uint4 hv = slot[k * kThreads];
        uint32_t w[4] = {hv.x, hv.y, hv.z, hv.w};
        const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&gw[j]));
          const __half2 o = __floats2half2_rn(x.x * inv * y.x, x.y * inv * y.y);
          w[j] = *reinterpret_cast<const uint32_t*>(&o);
        }
        slot[k * kThreads] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    hid = slot;
    return true;
  };

  // The next iteration's loads are issued as soon as the dot products have
  // consumed the rows, so the group's lane reductions and key updates run
  // while they are in flight.  Exception: the per-group fallback with the
  // fused norm enters a new row before issuing the loads, since the
  // normalisation needs registers that two rows in flight would occupy.
  const bool late_issue = kNorm && !table;
  while (c < c_end) {
    if (!pre && late_issue) {
      if (c >= row_e && !enter_row()) break;
      issue();
    }
    pre = false;
    if (c >= row_e && !enter_row()) break;
    const bool two = has1 && c + 1 < row_e;  // the second candidate is in this row
    // four partial sums per candidate (two per lane half of each 16-byte
    // chunk, alternating chunks): half the FMA dependency chain
    float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < kFastChunksPerLane; ++k) {
      const uint4 hk = hid[k * hstride];
      if (v0) dot_v4(a0[2 * (k & 1)], a0[2 * (k & 1) + 1], hk, e0[k]);
      if (v1) dot_v4(a1[2 * (k & 1)], a1[2 * (k & 1) + 1], hk, e1[k]);
    }
    const uint32_t id0 = t0, id1 = t1;
    const bool ok0 = v0, ok1 = v1;
    const int64_t n_here = two ? 2 : 1;
    seen += n_here;
    c += n_here;
    if (!late_issue && c < c_end) {
      issue();
      pre = true;
    }
    const float s0 = group8_sum((a0[0] + a0[1]) + (a0[2] + a0[3]), gmask);
    const float s1 = group8_sum((a1[0] + a1[1]) + (a1[2] + a1[3]), gmask);
    best = umax64(best, ok0 ? make_key(s0, id0) : kKeyPoison);
    if (two) best = umax64(best, ok1 ? make_key(s1, id1) : kKeyPoison);
  }
  if (have_row) flush_row<RowMode::kCsr>(p, rows_tab, r, row_b, row_e, best, seen, sub, bs);
}

template <RowMode M, bool kFast, bool kNorm = false, bool kIds16 = false>
__global__ void __launch_bounds__(kThreads, 2)
ragged_head_kernel(RaggedParams p, int64_t chunk) {
  // Dynamic shared memory: DFA mode, rows + 1 starts then rows arc bases;
  // CSR fast path, the per-lane hidden slots then the block's row table
  // (kCsrFastSmem bytes).
  extern __shared__ __align__(16) int32_t smem_rows[];
  __shared__ uint32_t s_last;
  // Fast path: each lane parks its 9 chunks of the current hidden row (after
  // the fused norm, when there is one) in its own shared-memory slot
  // (strided by thread, so conflict-free) instead of 36 registers; only that
  // lane reads them, so no synchronisation.  The freed registers hold the
  // two embedding rows in flight without spills (18.7 against 19.5 us per
  // headline batch for the plain head).
  __shared__ uint4 s_hid_dfa[(kFast && M == RowMode::kDfa) ? kThreads * kFastChunksPerLane : 1];
  uint4* const s_hid = M == RowMode::kCsr ? reinterpret_cast<uint4*>(smem_rows) : s_hid_dfa;

  Rows<M> rows_tab;
  int64_t total;
  __shared__ uint32_t s_row_counts[kThreads / 32][2];
  if (M == RowMode::kCsr) {
    // Overlapped launches: the next batch's blocks may start as this one's
    // retire.  Reads of this call's inputs need no wait (the caller promises
    // the previous kernel does not write them); every write waits (pdl_wait
    // in flush_row and before the epilogue below).
    pdl_trigger();
    rows_tab.start = p.offsets;
    total = p.total;
    // (the fast path checks inside csr_fast_block, behind its first loads)
    if (!kFast && p.rows <= kLocalCheckRows) {
      uint32_t first, last;  // (only the fast path uses the block's rows)
      if (!csr_local_check(p, min(p.total, (int64_t)blockIdx.x * kGroupsPerBlock * chunk),
                           min(p.total, (int64_t)(blockIdx.x + 1) * kGroupsPerBlock * chunk),
                           s_row_counts, first, last)) {
        csr_malformed(p);
        return;
      }
    }
  } else {
    pdl_trigger();  // the next decode step's blocks may queue behind this one's
    pdl_wait();     // a decode step reads the states the previous step wrote
    // Allowed-set lookup: per-sequence candidate counts from the DFA, and
    // their exclusive prefix sum in shared memory (every block computes the
    // same table).  Invalid states and empty sets get the sentinel.
    const uint32_t rows = p.rows;
    for (uint32_t r = threadIdx.x; r < rows; r += kThreads) {
      const bool owner = (r % gridDim.x) == blockIdx.x;
      uint32_t st;
      if (p.dfa_keys_in != nullptr) {
        // the previous step's result for row r, from its merged key: token
        // and next state packed in the id; no result keeps the state
        const unsigned long long k = __ldcg(p.dfa_keys_in + r);
        const uint32_t sp = p.states_prev[r];
        const bool res = key_is_result(k);
        st = res ? (key_id(k) & 0xFFFFu) : sp;
        if (owner) {
          p.prev_out_ids[r] = res ? key_id(k) >> 16 : kInvalid;
          if (p.prev_out_scores) p.prev_out_scores[r] = res ? key_score(k) : __uint_as_float(0x7FC00000u);
          p.states_in_w[r] = st;
        }
      } else {
        st = p.states_in[r];
      }
      if (p.dfa_keys_out != nullptr && owner) p.dfa_keys_clear[r] = 0ull;
      int32_t len = 0, base = 0;
      if (st < p.num_states) {
        const int32_t b = p.state_offsets[st], e = p.state_offsets[st + 1];
        if (b >= 0 && e > b && (int64_t)e <= p.num_arcs) len = e - b, base = b;
      }
      smem_rows[r + 1] = len;
      smem_rows[rows + 1 + r] = base;
      if (len == 0 && owner && p.dfa_keys_out == nullptr) {  // (keys mode: key 0 says so)
        p.out_ids[r] = kInvalid;
        p.states_out[r] = st;
        if (p.out_scores) p.out_scores[r] = __uint_as_float(0x7FC00000u);
      }
    }
    if (threadIdx.x == 0) smem_rows[0] = 0;
    __syncthreads();
    // inclusive scan of smem_rows[1..rows] (serial per warp chunk is fine
    // for <= 8192 rows: one warp scans, 32 lanes x chunks)
    if (threadIdx.x < 32) {
      const uint32_t per = (rows + 31) / 32;
      const uint32_t b = 1 + threadIdx.x * per;
      const uint32_t e = min(rows + 1, b + per);
      int32_t run = 0;
      for (uint32_t i = b; i < e; ++i) run += smem_rows[i];
      int32_t incl = run;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if ((int)threadIdx.x >= o) incl += v;
      }
      int32_t acc = incl - run;
      for (uint32_t i = b; i < e; ++i) {
        acc += smem_rows[i];
        smem_rows[i] = acc;
      }
    }
    __syncthreads();
    rows_tab.start = smem_rows;
    if constexpr (M == RowMode::kDfa) rows_tab.arc_base = smem_rows + rows + 1;
    total = smem_rows[rows];
    const int64_t groups = (int64_t)gridDim.x * kGroupsPerBlock;
    // as few candidates per group as the grid allows (at least one): a
    // step is a chain of dependent loads, so spreading a small step over
    // more groups shortens it (market grammar, B = 256: 8.0 to 5.0 us with
    // a floor of 1 instead of 4)
    chunk = (total + groups - 1) / groups;
    if (chunk < 1) chunk = 1;
  }

  __shared__ unsigned long long s_slot_key[kGroupsPerBlock];
  __shared__ uint32_t s_slot_count[kGroupsPerBlock];
  if (threadIdx.x < kGroupsPerBlock) {
    s_slot_key[threadIdx.x] = 0ull;
    s_slot_count[threadIdx.x] = 0u;
  }
  __syncthreads();
  BlockSlots bs;
  bs.key = s_slot_key;
  bs.count = s_slot_count;
  bs.chunk = chunk;
  bs.begin = min(total, (int64_t)blockIdx.x * kGroupsPerBlock * chunk);
  bs.end = min(total, bs.begin + (int64_t)kGroupsPerBlock * chunk);

  const int lane = threadIdx.x & 31;
  const int sub = lane & 7;
  const unsigned gmask = 0xFFu << (lane & ~7);
  const int64_t group = (int64_t)blockIdx.x * kGroupsPerBlock + (threadIdx.x >> 3);
  const int64_t c_begin = group * chunk;
  const int64_t c_end = min(total, c_begin + chunk);

  if (M == RowMode::kCsr && kFast) {
    __shared__ uint32_t s_rows_found[2];
    __shared__ int64_t s_tab_start[kBlockRows + 1];
    BlockRowTable tab;
    tab.rows = s_hid + kThreads * kFastChunksPerLane;  // after the per-lane slots
    tab.start = s_tab_start;
    csr_fast_block<kNorm, kIds16>(p, *reinterpret_cast<const Rows<RowMode::kCsr>*>(&rows_tab), c_begin,
                          c_end, sub, gmask, s_hid + threadIdx.x, bs, tab, s_rows_found,
                          s_row_counts);
  } else if (c_begin < c_end) {
    uint32_t r = find_row<M>(rows_tab, p.rows, c_begin, sub, gmask);
    int64_t row_b = rows_tab.at(r);
    int64_t row_e = rows_tab.at(r + 1);
    int64_t arc_base = 0;  // DFA: flat index -> arc index offset
    if constexpr (M == RowMode::kDfa) arc_base = (int64_t)rows_tab.arc_base[r] - row_b;

    float inv = 1.f;  // generic path: the row's inv_rms when normalising
    if (kFast) {
      stage_hidden_fast<kNorm>(p.hidden, r, sub, gmask, p.gamma, p.eps, s_hid + threadIdx.x);
    } else if (kNorm) {
      inv = row_inv_rms(p, r, sub, gmask);
    }
    unsigned long long best = kKeyNone;
    int64_t seen = 0;

    for (int64_t c = c_begin; c < c_end;) {
      // advance to the row that holds c (rows with no candidates are skipped)
      if (c >= row_e) {
        flush_row<M>(p, rows_tab, r, row_b, row_e, best, seen, sub, bs);
        best = kKeyNone;
        seen = 0;
        while (c >= row_e && r + 1 < p.rows) {
          ++r;
          row_b = row_e;
          row_e = rows_tab.at(r + 1);
        }
        if (c >= row_e || c < row_b) break;  // malformed offsets: stop
        if constexpr (M == RowMode::kDfa) arc_base = (int64_t)rows_tab.arc_base[r] - row_b;
        if (kFast) {
          stage_hidden_fast<kNorm>(p.hidden, r, sub, gmask, p.gamma, p.eps, s_hid + threadIdx.x);
        } else if (kNorm) {
          inv = row_inv_rms(p, r, sub, gmask);
        }
      }
      // up to two candidates of this row per iteration
      constexpr int R = 2;
      const int64_t n_here = min(min(c_end, row_e) - c, (int64_t)R);
      uint32_t t[R], id[R];
      bool v[R];
#pragma unroll
      for (int j = 0; j < R; ++j) {
        t[j] = 0;
        if constexpr (M == RowMode::kCsr) {
          if (j < n_here)
            t[j] = kIds16 ? (uint32_t)__ldg(p.ids16 + c + j) : (uint32_t)__ldg(p.ids + c + j);
        } else if (j < n_here) {
          t[j] = (uint32_t)p.ids[arc_base + c + j];
        }
        v[j] = j < n_here && t[j] < p.vocab;
        if constexpr (M == RowMode::kCsr) {
          id[j] = t[j];
        } else if (p.dfa_packed) {
          // the next state is read beside the token (same latency); one out
          // of range becomes 0xFFFF, itself out of range for these tables
          const uint32_t nx = j < n_here ? p.arc_next[arc_base + c + j] : 0u;
          id[j] = (t[j] << 16) | (nx < 0xFFFFu ? nx : 0xFFFFu);
        } else {
          id[j] = (uint32_t)(c + j - row_b);
        }
      }
      float sc[R];
      if (kFast) {
        uint4 e[R][kFastChunksPerLane];
#pragma unroll
        for (int j = 0; j < R; ++j) {
          const uint4* row = reinterpret_cast<const uint4*>(p.embedding + (size_t)(v[j] ? t[j] : 0) * kFastHidden);
          if (v[j]) {
#pragma unroll
            for (int k = 0; k < kFastChunksPerLane; ++k) e[j][k] = ld_stream_v4(row + sub + 8 * k);
          }
        }
        float a[R][2];
#pragma unroll
        for (int j = 0; j < R; ++j) a[j][0] = a[j][1] = 0.f;
#pragma unroll
        for (int k = 0; k < kFastChunksPerLane; ++k) {
          const uint4 hk = s_hid[k * kThreads + threadIdx.x];
#pragma unroll
          for (int j = 0; j < R; ++j)
            if (v[j]) dot_v4(a[j][0], a[j][1], hk, e[j][k]);
        }
#pragma unroll
        for (int j = 0; j < R; ++j) sc[j] = group8_sum(a[j][0] + a[j][1], gmask);
      } else {
#pragma unroll
        for (int j = 0; j < R; ++j)
          sc[j] = (j < n_here && v[j]) ? group_dot_generic(p, r, t[j], inv, sub, gmask) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < n_here) best = umax64(best, v[j] ? make_key(sc[j], id[j]) : kKeyPoison);
      seen += n_here;
      c += n_here;
    }
    flush_row<M>(p, rows_tab, r, row_b, row_e, best, seen, sub, bs);
  }

  if constexpr (M == RowMode::kDfa) return;
  // Offsets checked on entry: the finishing kernel decodes every row key
  // (an empty row's key is zero, which decodes to the sentinel).
  if (csr_keys_only(p)) return;
  // Empty rows get the sentinel here (no group visits them).
  pdl_wait();
  if (p.rows <= kLocalCheckRows) {  // one block, offsets checked on entry
    for (uint32_t r = threadIdx.x; r < p.rows; r += kThreads) {
      if (p.offsets[r] == p.offsets[r + 1]) {
        p.out_ids[r] = kInvalid;
        if (p.out_scores) p.out_scores[r] = __uint_as_float(0x7FC00000u);
      }
    }
    return;
  }
  // Larger batches: decreasing offsets or a bad first/last offset flag the
  // batch for the last block out.
  for (uint32_t r = blockIdx.x * kThreads + threadIdx.x; r < p.rows; r += gridDim.x * kThreads) {
    const int32_t b = p.offsets[r], e = p.offsets[r + 1];
    if (e < b) {
      atomicOr(p.control + 1, 1u);
    } else if (e == b) {
      p.out_ids[r] = kInvalid;
      if (p.out_scores) p.out_scores[r] = __uint_as_float(0x7FC00000u);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 &&
      (p.offsets[0] != 0 || (int64_t)p.offsets[p.rows] != p.total)) {
    atomicOr(p.control + 1, 1u);
  }

  // Last block out (CSR mode; DFA offsets are built in-kernel and cannot be
  // malformed): if the batch was flagged malformed, give every row the
  // sentinel and clear the whole workspace; then reset the control words.
  // Every thread fences first so its atomics and result stores are ordered
  // before this block's arrival on the done counter (one fence at exit costs
  // less than fencing each store inside the loop).
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = (atomicAdd(p.control, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    const uint32_t anomaly = atomicAdd(p.control + 1, 0u);
    if (anomaly) {
      for (uint32_t r = threadIdx.x; r < p.rows; r += kThreads) {
        p.keys[r] = 0ull;
        p.counts[r] = 0u;
        p.out_ids[r] = kInvalid;
        if (p.out_scores) p.out_scores[r] = __uint_as_float(0x7FC00000u);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      p.control[1] = 0u;
      p.control[0] = 0u;
    }
  }
}

// CSR batches of up to kLocalCheckRows rows on more than one block: after the
// whole head grid (a programmatic dependent launch that waits for it), every row
// key to the id and score rows, and the key back to zero for the next call.
__global__ void csr_finish_kernel(unsigned long long* keys, uint32_t* out_ids, float* out_scores,
                                  uint32_t rows) {
  pdl_trigger();
  pdl_wait();
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const unsigned long long k = keys[r];
  keys[r] = 0ull;
  const bool res = key_is_result(k);
  out_ids[r] = res ? key_id(k) : kInvalid;
  if (out_scores) out_scores[r] = res ? key_score(k) : __uint_as_float(0x7FC00000u);
}

// The last step of a packed-key decode: its keys to the token / score /
// state rows, and every key buffer back to zero.
__global__ void dfa_finish_kernel(const unsigned long long* keys, const uint32_t* states_prev,
                                  uint32_t* out_ids, float* out_scores, uint32_t* states_out,
                                  unsigned long long* k0, unsigned long long* k1,
                                  unsigned long long* k2, uint32_t rows) {
  pdl_wait();
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const unsigned long long k = keys[r];
  const bool res = key_is_result(k);
  out_ids[r] = res ? key_id(k) >> 16 : kInvalid;
  if (out_scores) out_scores[r] = res ? key_score(k) : __uint_as_float(0x7FC00000u);
  states_out[r] = res ? (key_id(k) & 0xFFFFu) : states_prev[r];
  k0[r] = 0ull;
  k1[r] = 0ull;
  k2[r] = 0ull;
}

// ---------------------------------------------------------------------------
// Host side

struct DeviceInfo {
  int sms = 0;
  int blocks_per_sm[2][2] = {{0, 0}, {0, 0}};  // [mode][fast]
};

static DeviceInfo& device_info() {
  static DeviceInfo info[64];
  int dev = 0;
  cudaGetDevice(&dev);
  DeviceInfo& d = info[dev & 63];
  if (d.sms == 0) {
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &d.blocks_per_sm[0][0], ragged_head_kernel<RowMode::kCsr, false>, kThreads, 0);
    cudaFuncSetAttribute(ragged_head_kernel<RowMode::kCsr, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, kCsrFastSmem);
    cudaFuncSetAttribute(ragged_head_kernel<RowMode::kCsr, true, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, kCsrFastSmem);
    cudaFuncSetAttribute(ragged_head_kernel<RowMode::kCsr, true, false, true>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, kCsrFastSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &d.blocks_per_sm[0][1], ragged_head_kernel<RowMode::kCsr, true>, kThreads, kCsrFastSmem);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &d.blocks_per_sm[1][0], ragged_head_kernel<RowMode::kDfa, false>, kThreads, 4096);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &d.blocks_per_sm[1][1], ragged_head_kernel<RowMode::kDfa, true>, kThreads, 4096);
    for (auto& m : d.blocks_per_sm)
      for (int& b : m)
        if (b < 1) b = 1;
    // DFA mode keeps 2 x batch + 1 ints in shared memory (up to ~64 KB)
    const int dfa_smem = (2 * kMaxDfaBatch + 1) * (int)sizeof(int32_t);
    for (auto k : {ragged_head_kernel<RowMode::kDfa, false>, ragged_head_kernel<RowMode::kDfa, true>,
                   ragged_head_kernel<RowMode::kDfa, false, true>,
                   ragged_head_kernel<RowMode::kDfa, true, true>})
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dfa_smem);
  }
  return d;
}

}  // namespace mfb

using namespace mfb;

namespace {

mf_status ok() { return mf_status{MF_OK, 0}; }
mf_status fail(int32_t code, uint32_t detail = 0) { return mf_status{code, detail}; }

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
  if (a != 0 && b > UINT64_MAX / a) return false;
  *out = a * b;
  return true;
}

bool distinct(std::initializer_list<const void*> ptrs) {
  const void* seen[16];
  int n = 0;
  for (const void* p : ptrs) {
    if (p == nullptr) return false;
    for (int i = 0; i < n; ++i)
      if (seen[i] == p) return false;
    seen[n++] = p;
  }
  return true;
}

// Every buffer starts on a multiple of the widest element the kernels load
// from or store to it (2-byte halves, 4-byte ints, 8-byte keys); a
// misaligned pointer is invalid_argument, not a device fault.  Null passes
// (the callers check which buffers may be null).
bool aligned(std::initializer_list<std::pair<const void*, uintptr_t>> bufs) {
  for (const auto& b : bufs)
    if ((uintptr_t)b.first % b.second != 0) return false;
  return true;
}

bool fast_path(const void* hidden, const void* embedding, uint64_t hidden_size) {
  return hidden_size == (uint64_t)kFastHidden && ((uintptr_t)hidden % 16) == 0 &&
         ((uintptr_t)embedding % 16) == 0;
}

mf_status launch_status(cudaError_t e) {
  return e == cudaSuccess ? ok() : fail(MF_CUDA_BACKEND_FAILURE, (uint32_t)e);
}

}  // namespace

extern "C" uint64_t mf_head_workspace_bytes(uint64_t rows) {
  // keys u64[rows] + counts u32[rows] + control u32[4], 16-byte multiple
  const uint64_t b = rows * 12 + 16;
  return (b + 15) & ~15ull;
}

// the head's workspace, then three key buffers of the packed-key decode
extern "C" uint64_t mf_dfa_workspace_bytes(uint64_t batch) {
  return mf_head_workspace_bytes(batch) + 3 * batch * 8;
}

namespace {

void split_workspace(void* ws, uint64_t rows, RaggedParams& p) {
  char* b = static_cast<char*>(ws);
  p.keys = reinterpret_cast<unsigned long long*>(b);
  p.counts = reinterpret_cast<uint32_t*>(b + rows * 8);
  p.control = reinterpret_cast<uint32_t*>(b + rows * 12);
}

}  // namespace

static mf_status csr_head(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t rows, uint64_t hidden_size,
    uint64_t vocab, void* stream, const void* gamma, float eps, uint32_t launch_flags,
    bool clear_workspace = false, bool ids_u16 = false) {
  if (rows == 0 || hidden_size == 0 || vocab == 0 || stream == nullptr ||
      (launch_flags & ~MF_LAUNCH_OVERLAP_PREVIOUS) != 0)
    return fail(MF_INVALID_ARGUMENT);
  if (vocab > UINT32_MAX || hidden_size > UINT32_MAX || rows > (uint64_t)INT32_MAX - 1)
    return fail(MF_RESOURCE_LIMIT);
  uint64_t hb, eb, ob;
  if (!mul_ok(rows, hidden_size, &hb) || !mul_ok(hb, 2, &hb) ||
      !mul_ok(vocab, hidden_size, &eb) || !mul_ok(eb, 2, &eb) || !mul_ok(rows + 1, 4, &ob))
    return fail(MF_ARITHMETIC_OVERFLOW);
  const uint64_t id_size = ids_u16 ? 2 : 4;
  if (ids_u16 && (vocab > 65536 || gamma))  // ids would not fit 16 bits; no fused-norm variant
    return fail(MF_INVALID_ARGUMENT);
  if (ids_bytes % id_size != 0 || ids_bytes / id_size > (uint64_t)INT32_MAX)
    return fail(MF_INVALID_ARGUMENT);
  if (hidden_bytes != hb || embedding_bytes != eb || offsets_bytes != ob ||
      out_ids_bytes != rows * 4 || (out_scores && out_scores_bytes != rows * 4) ||
      workspace_bytes < mf_head_workspace_bytes(rows))
    return fail(MF_INVALID_ARGUMENT);
  if (!distinct({hidden, embedding, offsets, out_ids, workspace}) ||
      (ids_bytes && !distinct({ids, hidden, embedding, offsets, out_ids, workspace})) ||
      (out_scores && !distinct({out_scores, hidden, embedding, offsets, out_ids, workspace})))
    return fail(MF_INVALID_ARGUMENT);
  if (!aligned({{hidden, 2}, {embedding, 2}, {offsets, 4}, {ids, id_size}, {out_ids, 4},
                {out_scores, 4}, {workspace, 8}, {gamma, 2}}))
    return fail(MF_INVALID_ARGUMENT);

  RaggedParams p{};
  p.hidden = static_cast<const __half*>(hidden);
  p.embedding = static_cast<const __half*>(embedding);
  p.offsets = static_cast<const int32_t*>(offsets);
  if (ids_u16)
    p.ids16 = static_cast<const uint16_t*>(ids);
  else
    p.ids = static_cast<const int32_t*>(ids);
  p.total = (int64_t)(ids_bytes / id_size);
  p.out_ids = static_cast<uint32_t*>(out_ids);
  p.out_scores = static_cast<float*>(out_scores);
  p.rows = (uint32_t)rows;
  p.hidden_size = (uint32_t)hidden_size;
  p.vocab = (uint32_t)vocab;
  p.gamma = static_cast<const __half*>(gamma);
  p.eps = eps;
  split_workspace(workspace, rows, p);

  const bool fast = fast_path(hidden, embedding, hidden_size);
  DeviceInfo& d = device_info();
  const int64_t max_blocks = (int64_t)d.sms * d.blocks_per_sm[0][fast ? 1 : 0];
  // at least 2 candidates per group so tiny batches do not launch idle blocks
  // (a floor of 8 made a one-row launch with K = 512 or 4,096 walk 8
  // dependent iterations per group: 8.5 / 8.8 us against 5.3 / 6.0 us)
  int64_t blocks = (p.total + (int64_t)kGroupsPerBlock * 2 - 1) / ((int64_t)kGroupsPerBlock * 2);
  blocks = blocks < 1 ? 1 : (blocks > max_blocks ? max_blocks : blocks);
  const int64_t groups = blocks * kGroupsPerBlock;
  int64_t chunk = (p.total + groups - 1) / groups;
  if (chunk < 1) chunk = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = fast ? kCsrFastSmem : 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  if (launch_flags & MF_LAUNCH_OVERLAP_PREVIOUS) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e;
  // Allocation-free entry: its shared scratch is cleared only once every
  // argument has passed, so a rejected call leaves the device untouched.
  if (clear_workspace) {
    e = cudaMemsetAsync(workspace, 0, mf_head_workspace_bytes(rows), cfg.stream);
    if (e != cudaSuccess) return fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
  }
  if (ids_u16)  // (the u16 entry has no fused norm)
    e = fast ? cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kCsr, true, false, true>, p,
                                  chunk)
             : cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kCsr, false, false, true>, p,
                                  chunk);
  else if (fast && p.gamma)
    e = cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kCsr, true, true>, p, chunk);
  else if (fast)
    e = cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kCsr, true>, p, chunk);
  else if (p.gamma)
    e = cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kCsr, false, true>, p, chunk);
  else
    e = cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kCsr, false>, p, chunk);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e == cudaSuccess && rows <= (uint64_t)kLocalCheckRows && blocks > 1) {
    cudaLaunchConfig_t fin = {};
    fin.gridDim = dim3((unsigned)((rows + kThreads - 1) / kThreads), 1, 1);
    fin.blockDim = dim3(kThreads, 1, 1);
    fin.stream = cfg.stream;
    cudaLaunchAttribute fa[1];
    fa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    fa[0].val.programmaticStreamSerializationAllowed = 1;
    fin.attrs = fa;
    fin.numAttrs = 1;
    e = cudaLaunchKernelEx(&fin, csr_finish_kernel, p.keys, p.out_ids, p.out_scores, p.rows);
    if (e == cudaSuccess) e = cudaGetLastError();
  }
  return launch_status(e);
}

extern "C" mf_status mf_head_restricted_csr_f16(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t rows, uint64_t hidden_size,
    uint64_t vocab, void* stream) {
  return csr_head(hidden, hidden_bytes, embedding, embedding_bytes, offsets, offsets_bytes, ids,
                  ids_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes, workspace,
                  workspace_bytes, rows, hidden_size, vocab, stream, nullptr, 0.f, 0u);
}

extern "C" mf_status mf_head_restricted_csr_f16_ex(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t rows, uint64_t hidden_size,
    uint64_t vocab, uint32_t launch_flags, void* stream) {
  return csr_head(hidden, hidden_bytes, embedding, embedding_bytes, offsets, offsets_bytes, ids,
                  ids_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes, workspace,
                  workspace_bytes, rows, hidden_size, vocab, stream, nullptr, 0.f, launch_flags);
}

extern "C" mf_status mf_head_restricted_csr_u16ids_f16_ex(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t rows, uint64_t hidden_size,
    uint64_t vocab, uint32_t launch_flags, void* stream) {
  return csr_head(hidden, hidden_bytes, embedding, embedding_bytes, offsets, offsets_bytes, ids,
                  ids_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes, workspace,
                  workspace_bytes, rows, hidden_size, vocab, stream, nullptr, 0.f, launch_flags,
                  false, true);
}

extern "C" mf_status mf_head_restricted_csr_rmsnorm_f16(
    const void* hidden, uint64_t hidden_bytes, const void* gamma, uint64_t gamma_bytes, float eps,
    const void* embedding, uint64_t embedding_bytes, const void* offsets, uint64_t offsets_bytes,
    const void* ids, uint64_t ids_bytes, void* out_ids, uint64_t out_ids_bytes, void* out_scores,
    uint64_t out_scores_bytes, void* workspace, uint64_t workspace_bytes, uint64_t rows,
    uint64_t hidden_size, uint64_t vocab, void* stream) {
  // rms_norm_f32's own checks (src/cpu/operators.cpp:498-501): finite eps > 0
  if (!(eps > 0.f) || !(eps < 3.0e38f) || gamma == nullptr)
    return fail(MF_INVALID_ARGUMENT);
  if (gamma_bytes != hidden_size * 2 || (uintptr_t)gamma % 16 != 0) return fail(MF_INVALID_ARGUMENT);
  if (gamma == hidden || gamma == embedding || gamma == offsets || gamma == ids ||
      gamma == out_ids || gamma == out_scores || gamma == workspace)
    return fail(MF_INVALID_ARGUMENT);
  return csr_head(hidden, hidden_bytes, embedding, embedding_bytes, offsets, offsets_bytes, ids,
                  ids_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes, workspace,
                  workspace_bytes, rows, hidden_size, vocab, stream, gamma, eps, 0u);
}

namespace {

mf_status dfa_validate(const void* hidden, uint64_t hidden_bytes, const void* embedding,
                       uint64_t embedding_bytes, const void* state_offsets,
                       uint64_t state_offsets_bytes, const void* arc_tokens,
                       uint64_t arc_tokens_bytes, const void* arc_next, uint64_t arc_next_bytes,
                       uint64_t steps, uint64_t batch, uint64_t num_states, uint64_t hidden_size,
                       uint64_t vocab, void* stream) {
  if (batch == 0 || num_states == 0 || hidden_size == 0 || vocab == 0 || steps == 0 ||
      stream == nullptr)
    return fail(MF_INVALID_ARGUMENT);
  if (vocab > UINT32_MAX || num_states > (uint64_t)INT32_MAX - 1 || hidden_size > UINT32_MAX ||
      batch > (uint64_t)kMaxDfaBatch)
    return fail(MF_RESOURCE_LIMIT);
  uint64_t hb, eb;
  if (!mul_ok(batch, hidden_size, &hb) || !mul_ok(hb, 2, &hb) || !mul_ok(hb, steps, &hb) ||
      !mul_ok(vocab, hidden_size, &eb) || !mul_ok(eb, 2, &eb))
    return fail(MF_ARITHMETIC_OVERFLOW);
  if (hidden_bytes != hb || embedding_bytes != eb || state_offsets_bytes != (num_states + 1) * 4 ||
      arc_tokens_bytes == 0 || arc_tokens_bytes % 4 != 0 || arc_next_bytes != arc_tokens_bytes ||
      arc_tokens_bytes / 4 > (uint64_t)INT32_MAX)
    return fail(MF_INVALID_ARGUMENT);
  if (!distinct({hidden, embedding, state_offsets, arc_tokens, arc_next}) ||
      !aligned({{hidden, 2}, {embedding, 2}, {state_offsets, 4}, {arc_tokens, 4}, {arc_next, 4}}))
    return fail(MF_INVALID_ARGUMENT);
  return ok();
}

// `after_step`: the previous kernel on `s` is the previous decode step, so
// this step launches as its programmatic dependent (its blocks take SM
// slots as the previous step's retire and wait in griddepcontrol.wait).
cudaError_t dfa_launch(RaggedParams p, bool fast, cudaStream_t s, bool after_step) {
  DeviceInfo& d = device_info();
  const int64_t blocks = (int64_t)d.sms * d.blocks_per_sm[1][fast ? 1 : 0];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (2 * (size_t)p.rows + 1) * sizeof(int32_t);  // <= 64 KB
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (after_step) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e;
  if (p.gamma != nullptr)
    e = fast ? cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kDfa, true, true>, p, (int64_t)0)
             : cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kDfa, false, true>, p,
                                  (int64_t)0);
  else
    e = fast ? cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kDfa, true>, p, (int64_t)0)
             : cudaLaunchKernelEx(&cfg, ragged_head_kernel<RowMode::kDfa, false>, p, (int64_t)0);
  return e == cudaSuccess ? cudaGetLastError() : e;
}

}  // namespace

static mf_status dfa_step(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* state_offsets, uint64_t state_offsets_bytes, const void* arc_tokens,
    uint64_t arc_tokens_bytes, const void* arc_next, uint64_t arc_next_bytes,
    const void* states_in, uint64_t states_in_bytes, void* states_out, uint64_t states_out_bytes,
    void* out_tokens, uint64_t out_tokens_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t batch, uint64_t num_states,
    uint64_t hidden_size, uint64_t vocab, void* stream, const void* gamma, float eps) {
  mf_status st = dfa_validate(hidden, hidden_bytes, embedding, embedding_bytes, state_offsets,
                              state_offsets_bytes, arc_tokens, arc_tokens_bytes, arc_next,
                              arc_next_bytes, 1, batch, num_states, hidden_size, vocab, stream);
  if (st.code != MF_OK) return st;
  if (states_in_bytes != batch * 4 || states_out_bytes != batch * 4 ||
      out_tokens_bytes != batch * 4 || (out_scores && out_scores_bytes != batch * 4) ||
      workspace_bytes < mf_head_workspace_bytes(batch) ||  // one step: no key buffers
      !distinct({states_in, states_out, out_tokens, workspace, hidden, embedding}) ||
      (out_scores && !distinct({out_scores, states_in, states_out, out_tokens, workspace})) ||
      !aligned({{states_in, 4}, {states_out, 4}, {out_tokens, 4}, {out_scores, 4},
                {workspace, 8}, {gamma, 2}}))
    return fail(MF_INVALID_ARGUMENT);
  RaggedParams p{};
  p.hidden = static_cast<const __half*>(hidden);
  p.embedding = static_cast<const __half*>(embedding);
  p.ids = static_cast<const int32_t*>(arc_tokens);
  p.state_offsets = static_cast<const int32_t*>(state_offsets);
  p.arc_next = static_cast<const uint32_t*>(arc_next);
  p.states_in = static_cast<const uint32_t*>(states_in);
  p.states_out = static_cast<uint32_t*>(states_out);
  p.num_states = (uint32_t)num_states;
  p.num_arcs = (int64_t)(arc_tokens_bytes / 4);
  p.out_ids = static_cast<uint32_t*>(out_tokens);
  p.out_scores = static_cast<float*>(out_scores);
  p.rows = (uint32_t)batch;
  p.hidden_size = (uint32_t)hidden_size;
  p.vocab = (uint32_t)vocab;
  p.gamma = static_cast<const __half*>(gamma);
  p.eps = eps;
  p.dfa_packed = vocab <= 65536u && num_states < 65535u ? 1u : 0u;
  split_workspace(workspace, batch, p);
  return launch_status(dfa_launch(p, fast_path(hidden, embedding, hidden_size),
                                  static_cast<cudaStream_t>(stream), false));
}

extern "C" mf_status mf_dfa_head_step_f16(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* state_offsets, uint64_t state_offsets_bytes, const void* arc_tokens,
    uint64_t arc_tokens_bytes, const void* arc_next, uint64_t arc_next_bytes,
    const void* states_in, uint64_t states_in_bytes, void* states_out, uint64_t states_out_bytes,
    void* out_tokens, uint64_t out_tokens_bytes, void* out_scores, uint64_t out_scores_bytes,
    void* workspace, uint64_t workspace_bytes, uint64_t batch, uint64_t num_states,
    uint64_t hidden_size, uint64_t vocab, void* stream) {
  return dfa_step(hidden, hidden_bytes, embedding, embedding_bytes, state_offsets,
                  state_offsets_bytes, arc_tokens, arc_tokens_bytes, arc_next, arc_next_bytes,
                  states_in, states_in_bytes, states_out, states_out_bytes, out_tokens,
                  out_tokens_bytes, out_scores, out_scores_bytes, workspace, workspace_bytes, batch,
                  num_states, hidden_size, vocab, stream, nullptr, 0.f);
}

extern "C" mf_status mf_dfa_head_step_rmsnorm_f16(
    const void* hidden, uint64_t hidden_bytes, const void* gamma, uint64_t gamma_bytes, float eps,
    const void* embedding, uint64_t embedding_bytes, const void* state_offsets,
    uint64_t state_offsets_bytes, const void* arc_tokens, uint64_t arc_tokens_bytes,
    const void* arc_next, uint64_t arc_next_bytes, const void* states_in,
    uint64_t states_in_bytes, void* states_out, uint64_t states_out_bytes, void* out_tokens,
    uint64_t out_tokens_bytes, void* out_scores, uint64_t out_scores_bytes, void* workspace,
    uint64_t workspace_bytes, uint64_t batch, uint64_t num_states, uint64_t hidden_size,
    uint64_t vocab, void* stream) {
  // rms_norm_f32's own checks (src/cpu/operators.cpp:498-501): finite eps > 0
  if (!(eps > 0.f) || !(eps < 3.0e38f) || gamma == nullptr) return fail(MF_INVALID_ARGUMENT);
  if (gamma_bytes != hidden_size * 2 || (uintptr_t)gamma % 16 != 0) return fail(MF_INVALID_ARGUMENT);
  if (gamma == hidden || gamma == embedding || gamma == states_out || gamma == out_tokens ||
      gamma == out_scores || gamma == workspace)
    return fail(MF_INVALID_ARGUMENT);
  return dfa_step(hidden, hidden_bytes, embedding, embedding_bytes, state_offsets,
                  state_offsets_bytes, arc_tokens, arc_tokens_bytes, arc_next, arc_next_bytes,
                  states_in, states_in_bytes, states_out, states_out_bytes, out_tokens,
                  out_tokens_bytes, out_scores, out_scores_bytes, workspace, workspace_bytes, batch,
                  num_states, hidden_size, vocab, stream, gamma, eps);
}

extern "C" mf_status mf_dfa_decode_f16(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* state_offsets, uint64_t state_offsets_bytes, const void* arc_tokens,
    uint64_t arc_tokens_bytes, const void* arc_next, uint64_t arc_next_bytes, void* state_trace,
    uint64_t state_trace_bytes, void* token_trace, uint64_t token_trace_bytes, void* score_trace,
    uint64_t score_trace_bytes, void* workspace, uint64_t workspace_bytes, uint64_t steps,
    uint64_t batch, uint64_t num_states, uint64_t hidden_size, uint64_t vocab, void* stream) {
  mf_status st = dfa_validate(hidden, hidden_bytes, embedding, embedding_bytes, state_offsets,
                              state_offsets_bytes, arc_tokens, arc_tokens_bytes, arc_next,
                              arc_next_bytes, steps, batch, num_states, hidden_size, vocab, stream);
  if (st.code != MF_OK) return st;
  uint64_t tb;
  if (!mul_ok(steps, batch, &tb) || !mul_ok(tb, 4, &tb)) return fail(MF_ARITHMETIC_OVERFLOW);
  if (state_trace_bytes != tb + batch * 4 || token_trace_bytes != tb ||
      (score_trace && score_trace_bytes != tb) || workspace_bytes < mf_dfa_workspace_bytes(batch) ||
      !distinct({state_trace, token_trace, workspace, hidden, embedding}) ||
      (score_trace && !distinct({score_trace, state_trace, token_trace, workspace})) ||
      !aligned({{state_trace, 4}, {token_trace, 4}, {score_trace, 4}, {workspace, 8}}))
    return fail(MF_INVALID_ARGUMENT);
  const bool fast = fast_path(hidden, embedding, hidden_size);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // packed keys (16-bit vocabulary and grammar): steps hand their results on
  // through three rotating key buffers after the head's workspace
  const bool packed = vocab <= 65536u && num_states < 65535u;
  unsigned long long* kbuf[3];
  for (int i = 0; i < 3; ++i)
    kbuf[i] = reinterpret_cast<unsigned long long*>(static_cast<char*>(workspace) +
                                                    mf_head_workspace_bytes(batch)) +
              (size_t)i * batch;
  for (uint64_t step = 0; step < steps; ++step) {
    RaggedParams p{};
    p.hidden = static_cast<const __half*>(hidden) + step * batch * hidden_size;
    p.embedding = static_cast<const __half*>(embedding);
    p.ids = static_cast<const int32_t*>(arc_tokens);
    p.state_offsets = static_cast<const int32_t*>(state_offsets);
    p.arc_next = static_cast<const uint32_t*>(arc_next);
    p.states_in = static_cast<const uint32_t*>(state_trace) + step * batch;
    p.states_out = static_cast<uint32_t*>(state_trace) + (step + 1) * batch;
    p.num_states = (uint32_t)num_states;
    p.num_arcs = (int64_t)(arc_tokens_bytes / 4);
    p.out_ids = static_cast<uint32_t*>(token_trace) + step * batch;
    p.out_scores = score_trace ? static_cast<float*>(score_trace) + step * batch : nullptr;
    p.rows = (uint32_t)batch;
    p.hidden_size = (uint32_t)hidden_size;
    p.vocab = (uint32_t)vocab;
    p.dfa_packed = packed ? 1u : 0u;
    split_workspace(workspace, batch, p);
    if (packed) {
      p.dfa_keys_out = kbuf[step % 3];
      p.dfa_keys_clear = kbuf[(step + 1) % 3];
      if (step > 0) {
        p.dfa_keys_in = kbuf[(step - 1) % 3];
        p.states_prev = static_cast<const uint32_t*>(state_trace) + (step - 1) * batch;
        p.states_in_w = static_cast<uint32_t*>(state_trace) + step * batch;
        p.prev_out_ids = static_cast<uint32_t*>(token_trace) + (step - 1) * batch;
        p.prev_out_scores =
            score_trace ? static_cast<float*>(score_trace) + (step - 1) * batch : nullptr;
      }
    }
    const cudaError_t e = dfa_launch(p, fast, s, step > 0);
    if (e != cudaSuccess) return launch_status(e);
  }
  if (packed) {  // the last step's keys, decoded as the next step would have
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((batch + 255) / 256), 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const uint64_t last = steps - 1;
    cudaError_t e = cudaLaunchKernelEx(
        &cfg, dfa_finish_kernel, (const unsigned long long*)kbuf[last % 3],
        static_cast<const uint32_t*>(state_trace) + last * batch,
        static_cast<uint32_t*>(token_trace) + last * batch,
        score_trace ? static_cast<float*>(score_trace) + last * batch : (float*)nullptr,
        static_cast<uint32_t*>(state_trace) + steps * batch, kbuf[0], kbuf[1], kbuf[2],
        (uint32_t)batch);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return launch_status(e);
  }
  return ok();
}

// ---------------------------------------------------------------------------
// Allocation-free variant of mf_head_restricted_csr_f16 (no counterpart in
// the reference).  For callers that may not allocate device memory: the
// workspace is this fixed device array instead of a caller buffer.  Every
// GPU that loads the library holds it until the process exits.

static __device__ __align__(256) unsigned char g_noalloc_scratch[MF_NOALLOC_SCRATCH_BYTES];

namespace {

// Device address of g_noalloc_scratch on the current device.  In host code
// the array's name is only a stand-in, never a device pointer, so the
// address comes from cudaGetSymbolAddress, once per device (cached).
cudaError_t noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    addr[dev] = p;
  }
  *out = addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" mf_status mf_head_restricted_csr_f16_noalloc(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* offsets, uint64_t offsets_bytes, const void* ids, uint64_t ids_bytes,
    void* out_ids, uint64_t out_ids_bytes, void* out_scores, uint64_t out_scores_bytes,
    uint64_t rows, uint64_t hidden_size, uint64_t vocab, void* stream) {
  if (rows == 0 || stream == nullptr) return fail(MF_INVALID_ARGUMENT);
  if (rows > MF_NOALLOC_MAX_ROWS) return fail(MF_RESOURCE_LIMIT);
  void* scratch = nullptr;
  cudaError_t e = noalloc_scratch(&scratch);
  if (e != cudaSuccess) return fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
  const uint64_t bytes = mf_head_workspace_bytes(rows);  // <= MF_NOALLOC_SCRATCH_BYTES
  // csr_head validates every argument first and only then clears the part
  // of the scratch this call uses (the kernel needs its keys, counters and
  // control words at zero) before the launch, both on `stream`.
  return csr_head(hidden, hidden_bytes, embedding, embedding_bytes, offsets, offsets_bytes, ids,
                  ids_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes, scratch, bytes,
                  rows, hidden_size, vocab, stream, nullptr, 0.f, 0u, true);
}
