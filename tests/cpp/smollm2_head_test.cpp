// Drives marketforge::cuda::SmolLm2OutputHead (the tail of
// CudaSmolLm2::forward, src/cuda/smollm2.cu:459-501) the way the model
// would: the decoder's output rows on the device, the final norm weight and
// the tied embedding; restricted decode over device ids (more than the
// reference's 128-id cap), full-vocabulary decode, and grammar decode over a
// device-resident DFA for several tokens.  Inputs come from a binary file
// written by tests/test_cpp_api.py; the selected tokens go to an output
// file that the test checks against the CPU oracle.
//
// input  (little-endian): u64 H, V, rows, n_allowed, S, A, steps;
//        f16 hidden[steps][rows][H]; f16 gamma[H]; f16 embedding[V][H];
//        i32 allowed[n_allowed]; i32 state_offsets[S+1]; i32 arc_tokens[A];
//        i32 arc_next[A]; u32 initial_state
// output: u32 restricted, greedy, grammar_tokens[steps], grammar_states[steps]
#include <cstdint>
#include <cstdio>
#include <utility>
#include <vector>

#include <cuda_runtime_api.h>

#include "marketforge/cuda/cuda_stream.hpp"
#include "marketforge/cuda/device_buffer.hpp"
#include "marketforge/cuda/smollm2_head.hpp"

using namespace marketforge;
using namespace marketforge::cuda;

namespace {

template <typename T>
bool read(std::FILE* f, std::vector<T>& v, std::uint64_t n) {
  v.resize(n);
  return std::fread(v.data(), sizeof(T), n, f) == n;
}

bool upload(DeviceBuffer& b, const void* src, std::uint64_t bytes, StreamHandle s) {
  auto r = DeviceBuffer::allocate(bytes);
  if (!r) return false;
  b = std::move(r).value();
  return b.copy_from_host_async(src, bytes, 0, s).ok();
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 3) return 2;
  std::FILE* in = std::fopen(argv[1], "rb");
  if (!in) return 2;
  std::uint64_t hdr[7];
  if (std::fread(hdr, 8, 7, in) != 7) return 2;
  const std::uint64_t H = hdr[0], V = hdr[1], rows = hdr[2], n_allowed = hdr[3], S = hdr[4],
                      A = hdr[5], steps = hdr[6];
  std::vector<std::uint16_t> hidden, gamma, emb;
  std::vector<std::int32_t> allowed, off, tok, nxt;
  std::vector<std::uint32_t> init;
  if (!read(in, hidden, steps * rows * H) || !read(in, gamma, H) || !read(in, emb, V * H) ||
      !read(in, allowed, n_allowed) || !read(in, off, S + 1) || !read(in, tok, A) ||
      !read(in, nxt, A) || !read(in, init, 1))
    return 2;
  std::fclose(in);

  auto sr = CudaStream::create();
  if (!sr) return 3;
  CudaStream stream = std::move(sr).value();
  const StreamHandle s = stream.handle();
  std::vector<DeviceBuffer> hid(steps);
  DeviceBuffer g, e, a, so, at, an, state;
  for (std::uint64_t k = 0; k < steps; ++k)
    if (!upload(hid[k], hidden.data() + k * rows * H, rows * H * 2, s)) return 3;
  if (!upload(g, gamma.data(), H * 2, s) || !upload(e, emb.data(), V * H * 2, s) ||
      !upload(a, allowed.data(), n_allowed * 4, s) || !upload(so, off.data(), (S + 1) * 4, s) ||
      !upload(at, tok.data(), A * 4, s) || !upload(an, nxt.data(), A * 4, s) ||
      !upload(state, init.data(), 4, s))
    return 3;

  auto hr = SmolLm2OutputHead::create({H, V, 1.0e-5F}, s);
  if (!hr) return 4;
  SmolLm2OutputHead head = std::move(hr).value();
  std::vector<std::uint32_t> out;
  auto r1 = head.select_restricted(hid[0], rows, g, e, a, n_allowed, s);
  auto r2 = head.select_greedy(hid[0], rows, g, e, s);
  if (!r1 || !r2) return 5;
  out.push_back(r1.value());
  out.push_back(r2.value());
  std::vector<std::uint32_t> states;
  for (std::uint64_t k = 0; k < steps; ++k) {
    auto r = head.select_grammar(hid[k], rows, g, e, so, at, an, state, S, s);
    if (!r) return 6;
    out.push_back(r.value());
    std::uint32_t st = 0;
    if (!state.copy_to_host_async(&st, 4, 0, s).ok() || !stream.synchronize().ok()) return 6;
    states.push_back(st);
  }
  out.insert(out.end(), states.begin(), states.end());
  // a rejected call: wrong row count for the hidden buffer
  auto bad = head.select_greedy(hid[0], rows + 1, g, e, s);
  if (bad || bad.status().code != ErrorCode::invalid_argument) return 7;

  std::FILE* o = std::fopen(argv[2], "wb");
  if (!o) return 8;
  std::fwrite(out.data(), 4, out.size(), o);
  std::fclose(o);
  std::printf("SMOLLM2 HEAD OK\n");
  return 0;
}
