// C++ callers of the head, written against the reference's interface
// (marketforge::cuda, include/marketforge/cuda/greedy.hpp): the known-answer
// cases of the reference's tests/cuda/cuda_tests.cu restated, plus the new
// ragged, DFA and dense entry points.  Prints "ALL PASSED" and exits 0 on
// success.  Built and run by tests/test_cpp_api.py.
#include <cuda_fp16.h>

#include <array>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <limits>
#include <vector>

#include "marketforge/cuda/greedy.hpp"
#include "marketforge/cuda/restricted_head.hpp"
#include "mf_head.h"

using marketforge::ErrorCode;
using namespace marketforge::cuda;

static int failures = 0;
#define CHECK(c)                                                       \
  do {                                                                 \
    if (!(c)) {                                                        \
      std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #c);       \
      ++failures;                                                      \
    }                                                                  \
  } while (0)

template <typename T>
static DeviceBuffer upload(const std::vector<T>& v, const CudaStream& s) {
  auto b = DeviceBuffer::allocate(v.size() * sizeof(T));
  CHECK(b.has_value());
  DeviceBuffer d = std::move(b).value();
  CHECK(d.copy_from_host_async(v.data(), v.size() * sizeof(T), 0, s.handle()).ok());
  return d;
}

template <typename T>
static std::vector<T> download(const DeviceBuffer& d, size_t n, const CudaStream& s) {
  std::vector<T> v(n);
  CHECK(d.copy_to_host_async(v.data(), n * sizeof(T), 0, s.handle()).ok());
  CHECK(s.synchronize().ok());
  return v;
}

// cuda_tests.cu:699-800 — 3 x 8 x 17 with a tie (rows 4 and 6) and an all-NaN row.
static void restricted_head_kat(const CudaStream& s) {
  const uint64_t rows = 3, hs = 8, vocab = 17, mx = 5;
  std::vector<__half> hidden(rows * hs), emb(vocab * hs);
  for (size_t i = 0; i < hidden.size(); ++i) hidden[i] = __float2half_rn(float((int)(i % 11) - 5) / 8.f);
  for (size_t i = 0; i < emb.size(); ++i) emb[i] = __float2half_rn(float((int)((i * 7) % 19) - 9) / 16.f);
  for (uint64_t f = 0; f < hs; ++f) {
    emb[6 * hs + f] = emb[4 * hs + f];
    hidden[2 * hs + f] = __float2half_rn(std::numeric_limits<float>::quiet_NaN());
  }
  std::vector<uint32_t> allowed{9, 3, 14, 0, 0, 6, 4, 8, 0, 0, 7, 1, 0, 0, 0}, counts{3, 3, 2};
  std::vector<uint32_t> expected(rows);
  for (uint64_t r = 0; r < rows; ++r) {
    float best = -INFINITY;
    uint32_t win = restricted_greedy_invalid_token_id, fb = restricted_greedy_invalid_token_id;
    for (uint32_t k = 0; k < counts[r]; ++k) {
      const uint32_t t = allowed[r * mx + k];
      fb = t < fb ? t : fb;
      float sc = 0.f;
      for (uint64_t f = 0; f < hs; ++f)
        sc = std::fma(__half2float(hidden[r * hs + f]), __half2float(emb[t * hs + f]), sc);
      if (sc > best || (sc == best && t < win)) best = sc, win = t;
    }
    expected[r] = win != restricted_greedy_invalid_token_id ? win : fb;
  }
  auto h = upload(hidden, s), e = upload(emb, s), a = upload(allowed, s), c = upload(counts, s);
  auto out = std::move(DeviceBuffer::allocate(rows * 4)).value();
  CHECK(restricted_output_head_f16(h, e, a, c, out, rows, hs, vocab, mx, s.handle()).ok());
  CHECK(download<uint32_t>(out, rows, s) == expected);
  // cuda_tests.cu:1283-1339 — host rejections
  CHECK(restricted_output_head_f16(h, e, a, c, out, 0, hs, vocab, mx, s.handle()).code == ErrorCode::invalid_argument);
  CHECK(restricted_output_head_f16(h, e, a, c, out, rows, hs, vocab, 0, s.handle()).code == ErrorCode::invalid_argument);
  CHECK(restricted_output_head_f16(h, e, a, c, out, rows, hs, vocab, mx, {}).code == ErrorCode::invalid_argument);
  CHECK(restricted_output_head_f16(h, e, a, c, c, rows, hs, vocab, mx, s.handle()).code == ErrorCode::invalid_argument);
  CHECK(restricted_output_head_f16(h, e, a, c, out, UINT64_MAX, hs, vocab, mx, s.handle()).code == ErrorCode::resource_limit);
}

// cuda_tests.cu:1341-1404 — count 0, count > max, id >= V give the sentinel.
static void invalid_rows(const CudaStream& s) {
  std::vector<__half> hidden(3 * 2, __float2half_rn(0.f)), emb(5 * 2, __float2half_rn(0.f));
  std::vector<uint32_t> allowed{1, 2, 2, 3, 1, 5}, counts{0, 3, 2};
  auto h = upload(hidden, s), e = upload(emb, s), a = upload(allowed, s), c = upload(counts, s);
  auto out = std::move(DeviceBuffer::allocate(12)).value();
  CHECK(restricted_output_head_f16(h, e, a, c, out, 3, 2, 5, 2, s.handle()).ok());
  for (uint32_t t : download<uint32_t>(out, 3, s)) CHECK(t == restricted_greedy_invalid_token_id);
}

// cuda_tests.cu:508-565 — lowest-id ties and the NaN/-inf row, V = 17 and 49,152.
static void greedy_kat(const CudaStream& s, uint64_t rows, uint64_t vocab) {
  std::vector<__half> logits(rows * vocab, __float2half_rn(-4.f));
  std::vector<uint32_t> expected(rows);
  for (uint64_t r = 0; r < rows; ++r) {
    const uint64_t w = (r * 7 + 3) % vocab;
    expected[r] = (uint32_t)w;
    logits[r * vocab + w] = __float2half_rn(8.f);
  }
  if (rows > 1 && vocab > 9) logits[vocab + 9] = __float2half_rn(8.f), expected[1] = 9;
  if (rows > 2) {
    for (uint64_t t = 0; t < vocab; ++t) logits[2 * vocab + t] = __float2half_rn(-INFINITY);
    logits[2 * vocab] = __float2half_rn(NAN);
    expected[2] = 1;
  }
  auto l = upload(logits, s);
  auto out = std::move(DeviceBuffer::allocate(rows * 4)).value();
  CHECK(greedy_select_f16(l, out, rows, vocab, s.handle()).ok());
  CHECK(download<uint32_t>(out, rows, s) == expected);
}

// The new entry points agree with each other: the ragged CSR head and the
// padded head pick the same ids; the dense head over a vocabulary equal to
// every row's allowed set picks the same ids as the ragged head over it.
static void new_entry_points(const CudaStream& s) {
  const uint64_t rows = 130, hs = 576, vocab = 1000;
  std::vector<__half> hidden(rows * hs), emb(vocab * hs);
  uint64_t x = 12345;
  auto rnd = [&] { x = x * 6364136223846793005ull + 1442695040888963407ull; return (double)(x >> 11) / 9007199254740992.0; };
  for (auto& v : hidden) v = __float2half_rn((float)(rnd() * 2 - 1));
  for (auto& v : emb) v = __float2half_rn((float)((rnd() * 2 - 1) * 0.05));
  std::vector<int32_t> offsets(rows + 1), ids;
  for (uint64_t r = 0; r < rows; ++r) {
    offsets[r] = (int32_t)ids.size();
    for (uint32_t t = 0; t < vocab; ++t) ids.push_back((int32_t)t);  // everything allowed
  }
  offsets[rows] = (int32_t)ids.size();
  auto h = upload(hidden, s), e = upload(emb, s), o = upload(offsets, s), i = upload(ids, s);
  auto ws = std::move(allocate_head_workspace(rows, s.handle())).value();
  auto out = std::move(DeviceBuffer::allocate(rows * 4)).value();
  auto sc = std::move(DeviceBuffer::allocate(rows * 4)).value();
  CHECK(restricted_output_head_csr_f16(h, e, o, i, out, sc, ws, rows, hs, vocab, s.handle()).ok());
  const auto ragged = download<uint32_t>(out, rows, s);
  DeviceBuffer no_keys;
  CHECK(dense_output_head_f16(h, e, no_keys, out, ws, rows, hs, vocab, 0, s.handle()).ok());
  const auto dense = download<uint32_t>(out, rows, s);
  const auto scores = download<float>(sc, rows, s);
  int same = 0;
  for (uint64_t r = 0; r < rows; ++r) same += ragged[r] == dense[r];
  CHECK(same >= (int)rows - 2);  // FP32 summation order may flip a near-tie
  for (float v : scores) CHECK(std::isfinite(v));

  // overlapped back-to-back launches give the same ids as the plain call
  auto out2 = std::move(DeviceBuffer::allocate(rows * 4)).value();
  CHECK(restricted_output_head_csr_f16(h, e, o, i, out, sc, ws, rows, hs, vocab,
                                       launch_overlap_previous, s.handle()).ok());
  CHECK(restricted_output_head_csr_f16(h, e, o, i, out2, sc, ws, rows, hs, vocab,
                                       launch_overlap_previous, s.handle()).ok());
  CHECK(download<uint32_t>(out, rows, s) == ragged);
  CHECK(download<uint32_t>(out2, rows, s) == ragged);

  // the sharded dense head with one rank (its own exchange buffer) equals the dense head
  auto xb = std::move(DeviceBuffer::allocate(mf_exchange_bytes(rows, 1))).value();
  void* exchange[1] = {reinterpret_cast<void*>(xb.address().value)};
  CHECK(dense_output_head_sharded_f16(h, e, no_keys, out, ws, rows, hs, vocab, 0, exchange,
                                      xb.size_bytes(), 1, 0, s.handle()).ok());
  CHECK(download<uint32_t>(out, rows, s) == dense);
}

int main() {
  auto sr = CudaStream::create();
  if (!sr) {
    std::printf("no CUDA stream (code %d)\n", (int)sr.status().code);
    return 2;
  }
  CudaStream s = std::move(sr).value();
  restricted_head_kat(s);
  invalid_rows(s);
  greedy_kat(s, 1, 17);
  greedy_kat(s, 3, 49152);
  new_entry_points(s);
  if (failures) {
    std::printf("%d FAILED\n", failures);
    return 1;
  }
  std::printf("ALL PASSED\n");
  return 0;
}
