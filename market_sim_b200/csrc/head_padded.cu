// Reference-signature entry points that need no workspace:
//   mf_restricted_output_head_f16   (src/cuda/greedy.cu:133-212, 349-414)
//   mf_restricted_greedy_select_f16 (src/cuda/greedy.cu:61-131, 281-347)
//   mf_greedy_select_f16            (src/cuda/greedy.cu:21-59, 237-279)
//
// The padded head keeps the reference's "one row, no workspace" contract: a
// row is owned by one thread block, or, for long candidate tables (more than
// 512 ids per row), by a thread-block cluster of up to 8 CTAs that split the
// row's candidates and merge their keys through distributed shared memory
// (still no global scratch).  Inside a block
// the work is laid out for B200: 32 groups of 8 lanes, each group reading
// one 1152-byte embedding row as 9 coalesced 16-byte loads per lane (two
// rows in flight), fp16 x fp16 -> f32 FMAs, a shuffle dot reduction and a
// packed-key argmax (see common.cuh for the key order).
#include <cuda_runtime.h>

#include <initializer_list>
#include <utility>

#include "common.cuh"

namespace mfb {

constexpr int kRowThreads = 256;
constexpr int kRowGroups = kRowThreads / 8;

__device__ unsigned long long block_max_key(unsigned long long k) {
  __shared__ unsigned long long part[kRowThreads / 32];
  k = warp_max_key(k);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) part[warp] = k;
  __syncthreads();
  if (threadIdx.x < 32) {
    k = threadIdx.x < kRowThreads / 32 ? part[threadIdx.x] : 0ull;
    k = warp_max_key(k);
  }
  return k;  // valid in warp 0
}

// kCluster: launched with a cluster dimension C (grid = rows x C); CTA k of
// the cluster takes the row's candidate groups k, k + C, ... and rank 0
// merges the C block keys read from the peers' shared memory.
template <bool kFast, bool kCluster = false>
__global__ void __launch_bounds__(kRowThreads)
padded_head_kernel(const __half* __restrict__ hidden, const __half* __restrict__ emb,
                   const uint32_t* __restrict__ allowed, const uint32_t* __restrict__ counts,
                   uint32_t* __restrict__ out, uint32_t width, uint32_t vocab, uint64_t max_allowed) {
  uint32_t crank = 0, csize = 1;
  if (kCluster) {
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
    asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(csize));
  }
  const uint32_t r = blockIdx.x / csize;
  const uint64_t n = counts[r];
  const bool row_bad = n == 0 || n > max_allowed;
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const unsigned gmask = 0xFFu << (lane & ~7);
  const int g = (int)(crank * kRowGroups) + (threadIdx.x >> 3);  // group within the row's cluster
  const uint64_t gstride = (uint64_t)kRowGroups * csize;
  const uint32_t* cand = allowed + (uint64_t)r * max_allowed;
  unsigned long long best = 0ull;
  if (!row_bad) {
    uint4 h[kFast ? kFastChunksPerLane : 1];
    if (kFast) {
      const uint4* hr = reinterpret_cast<const uint4*>(hidden + (size_t)r * kFastHidden);
#pragma unroll
      for (int k = 0; k < kFastChunksPerLane; ++k) h[k] = ld_v4(hr + sub + 8 * k);
    }
    for (uint64_t i = g; i < n; i += 2 * gstride) {
      const bool two = i + gstride < n;
      const uint32_t t0 = cand[i];
      const uint32_t t1 = two ? cand[i + gstride] : 0u;
      const bool v0 = t0 < vocab, v1 = two && t1 < vocab;
      float s0 = 0.f, s1 = 0.f;
      if (kFast) {
        uint4 e0[kFastChunksPerLane], e1[kFastChunksPerLane];
        const uint4* r0 = reinterpret_cast<const uint4*>(emb + (size_t)(v0 ? t0 : 0) * kFastHidden);
        const uint4* r1 = reinterpret_cast<const uint4*>(emb + (size_t)(v1 ? t1 : 0) * kFastHidden);
        if (v0) {
#pragma unroll
          for (int k = 0; k < kFastChunksPerLane; ++k) e0[k] = ld_stream_v4(r0 + sub + 8 * k);
        }
        if (v1) {
#pragma unroll
          for (int k = 0; k < kFastChunksPerLane; ++k) e1[k] = ld_stream_v4(r1 + sub + 8 * k);
        }
        float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
        if (v0) {
#pragma unroll
          for (int k = 0; k < kFastChunksPerLane; ++k) dot_v4(a0, a1, h[k], e0[k]);
        }
        if (v1) {
#pragma unroll
          for (int k = 0; k < kFastChunksPerLane; ++k) dot_v4(b0, b1, h[k], e1[k]);
        }
        s0 = group8_sum(a0 + a1, gmask);
        s1 = group8_sum(b0 + b1, gmask);
      } else {
        const __half* hr = hidden + (size_t)r * width;
        float a = 0.f, b = 0.f;
        if (v0)
          for (uint32_t f = sub; f < width; f += 8)
            a = fmaf(__half2float(hr[f]), __half2float(emb[(size_t)t0 * width + f]), a);
        if (v1)
          for (uint32_t f = sub; f < width; f += 8)
            b = fmaf(__half2float(hr[f]), __half2float(emb[(size_t)t1 * width + f]), b);
        s0 = group8_sum(a, gmask);
        s1 = group8_sum(b, gmask);
      }
      best = umax64(best, v0 ? make_key(s0, t0) : kKeyPoison);
      if (two) best = umax64(best, v1 ? make_key(s1, t1) : kKeyPoison);
    }
  }
  best = block_max_key(best);
  if (kCluster) {
    // merge the cluster's block keys in rank 0 through distributed shared
    // memory; the second barrier keeps every peer's key alive until read
    __shared__ unsigned long long s_key;
    if (threadIdx.x == 0) s_key = best;
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
    if (crank == 0 && threadIdx.x == 0) {
      const uint32_t local = (uint32_t)__cvta_generic_to_shared(&s_key);
      for (uint32_t q = 1; q < csize; ++q) {
        uint32_t remote;
        unsigned long long k;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(q));
        asm volatile("ld.shared::cluster.u64 %0, [%1];" : "=l"(k) : "r"(remote) : "memory");
        best = umax64(best, k);
      }
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
    if (crank != 0) return;
  }
  if (threadIdx.x == 0) out[r] = (!row_bad && key_is_result(best)) ? key_id(best) : kInvalid;
}

// Masked argmax over materialised fp16 logits: one warp per row.
__global__ void __launch_bounds__(256)
restricted_select_kernel(const __half* __restrict__ logits, const uint32_t* __restrict__ allowed,
                         const uint32_t* __restrict__ counts, uint32_t* __restrict__ out,
                         uint32_t rows, uint64_t vocab, uint64_t max_allowed) {
  const uint32_t r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const uint64_t n = counts[r];
  const bool row_bad = n == 0 || n > max_allowed;
  unsigned long long best = 0ull;
  if (!row_bad) {
    const uint32_t* cand = allowed + (uint64_t)r * max_allowed;
    const __half* lr = logits + (uint64_t)r * vocab;
    for (uint64_t i = lane; i < n; i += 32) {
      const uint32_t t = cand[i];
      best = umax64(best, t < vocab ? make_key(__half2float(lr[t]), t) : kKeyPoison);
    }
  }
  best = warp_max_key(best);
  if (lane == 0) out[r] = (!row_bad && key_is_result(best)) ? key_id(best) : kInvalid;
}

// Full-row argmax over fp16 logits: one block per row, 16-byte loads when
// the row is 16-byte aligned.  An all-NaN row gives the lowest NaN id, i.e.
// token 0, which is the reference's fallback.
__global__ void __launch_bounds__(kRowThreads)
greedy_kernel(const __half* __restrict__ logits, uint32_t* __restrict__ out, uint64_t vocab,
              bool vec) {
  const uint32_t r = blockIdx.x;
  const __half* lr = logits + (uint64_t)r * vocab;
  unsigned long long best = 0ull;
  if (vec) {
    const uint4* v = reinterpret_cast<const uint4*>(lr);
    for (uint64_t i = threadIdx.x; i < vocab / 8; i += kRowThreads) {
      const uint4 q = ld_stream_v4(v + i);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 h2 = *reinterpret_cast<const __half2*>(&w[j]);
        const float2 f = __half22float2(h2);
        best = umax64(best, make_key(f.x, (uint32_t)(i * 8 + 2 * j)));
        best = umax64(best, make_key(f.y, (uint32_t)(i * 8 + 2 * j + 1)));
      }
    }
  } else {
    for (uint64_t i = threadIdx.x; i < vocab; i += kRowThreads)
      best = umax64(best, make_key(__half2float(lr[i]), (uint32_t)i));
  }
  best = block_max_key(best);
  if (threadIdx.x == 0) out[r] = key_is_result(best) ? key_id(best) : 0u;
}

}  // namespace mfb

using namespace mfb;

namespace {

mf_status ok() { return mf_status{MF_OK, 0}; }
mf_status fail(int32_t code, uint32_t detail = 0) { return mf_status{code, detail}; }
mf_status launch_status(cudaError_t e) {
  return e == cudaSuccess ? ok() : fail(MF_CUDA_BACKEND_FAILURE, (uint32_t)e);
}
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
// Every buffer starts on a multiple of the widest element the kernels
// access in it: a misaligned pointer is invalid_argument, not a device fault.
bool aligned(std::initializer_list<std::pair<const void*, uintptr_t>> bufs) {
  for (const auto& b : bufs)
    if ((uintptr_t)b.first % b.second != 0) return false;
  return true;
}

}  // namespace

extern "C" uint32_t mf_version(void) { return 1u; }
extern "C" uint32_t mf_built_arch(void) { return 1000u; }

// src/cuda/greedy.cu:237-279
extern "C" mf_status mf_greedy_select_f16(const void* logits, uint64_t logits_bytes,
                                          void* token_ids, uint64_t token_ids_bytes, uint64_t rows,
                                          uint64_t vocab, void* stream) {
  if (rows == 0 || vocab == 0 || stream == nullptr) return fail(MF_INVALID_ARGUMENT);
  if (vocab > UINT32_MAX) return fail(MF_RESOURCE_LIMIT);
  if (rows > (uint64_t)INT32_MAX) return fail(MF_RESOURCE_LIMIT);
  uint64_t elems, lb, tb;
  if (!mul_ok(rows, vocab, &elems) || !mul_ok(elems, 2, &lb) || !mul_ok(rows, 4, &tb))
    return fail(MF_ARITHMETIC_OVERFLOW);
  if (logits_bytes != lb || token_ids_bytes != tb || !distinct({logits, token_ids}) ||
      !aligned({{logits, 2}, {token_ids, 4}}))
    return fail(MF_INVALID_ARGUMENT);
  const bool vec = vocab % 8 == 0 && (uintptr_t)logits % 16 == 0;
  greedy_kernel<<<(unsigned)rows, kRowThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(logits), static_cast<uint32_t*>(token_ids), vocab, vec);
  return launch_status(cudaGetLastError());
}

// src/cuda/greedy.cu:281-347
extern "C" mf_status mf_restricted_greedy_select_f16(
    const void* logits, uint64_t logits_bytes, const void* allowed, uint64_t allowed_bytes,
    const void* counts, uint64_t counts_bytes, void* token_ids, uint64_t token_ids_bytes,
    uint64_t rows, uint64_t vocab, uint64_t max_allowed, void* stream) {
  if (rows == 0 || vocab == 0 || max_allowed == 0 || stream == nullptr)
    return fail(MF_INVALID_ARGUMENT);
  if (vocab > UINT32_MAX || max_allowed > UINT32_MAX || rows > (uint64_t)INT32_MAX)
    return fail(MF_RESOURCE_LIMIT);
  uint64_t le, ae, lb, ab, rb;
  if (!mul_ok(rows, vocab, &le) || !mul_ok(rows, max_allowed, &ae) || !mul_ok(le, 2, &lb) ||
      !mul_ok(ae, 4, &ab) || !mul_ok(rows, 4, &rb))
    return fail(MF_ARITHMETIC_OVERFLOW);
  if (logits_bytes != lb || allowed_bytes != ab || counts_bytes != rb || token_ids_bytes != rb ||
      !distinct({logits, allowed, counts, token_ids}) ||
      !aligned({{logits, 2}, {allowed, 4}, {counts, 4}, {token_ids, 4}}))
    return fail(MF_INVALID_ARGUMENT);
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  restricted_select_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(logits), static_cast<const uint32_t*>(allowed),
      static_cast<const uint32_t*>(counts), static_cast<uint32_t*>(token_ids), (uint32_t)rows,
      vocab, max_allowed);
  return launch_status(cudaGetLastError());
}

// src/cuda/greedy.cu:349-414
extern "C" mf_status mf_restricted_output_head_f16(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    const void* allowed, uint64_t allowed_bytes, const void* counts, uint64_t counts_bytes,
    void* token_ids, uint64_t token_ids_bytes, uint64_t rows, uint64_t hidden_size,
    uint64_t vocab, uint64_t max_allowed, void* stream) {
  if (rows == 0 || hidden_size == 0 || vocab == 0 || max_allowed == 0 || stream == nullptr)
    return fail(MF_INVALID_ARGUMENT);
  if (vocab > UINT32_MAX || max_allowed > UINT32_MAX || rows > (uint64_t)INT32_MAX)
    return fail(MF_RESOURCE_LIMIT);
  uint64_t he, ee, ae, hb, eb, ab, rb;
  if (!mul_ok(rows, hidden_size, &he) || !mul_ok(vocab, hidden_size, &ee) ||
      !mul_ok(rows, max_allowed, &ae) || !mul_ok(he, 2, &hb) || !mul_ok(ee, 2, &eb) ||
      !mul_ok(ae, 4, &ab) || !mul_ok(rows, 4, &rb))
    return fail(MF_ARITHMETIC_OVERFLOW);
  if (hidden_bytes != hb || embedding_bytes != eb || allowed_bytes != ab || counts_bytes != rb ||
      token_ids_bytes != rb || !distinct({hidden, embedding, allowed, counts, token_ids}) ||
      !aligned({{hidden, 2}, {embedding, 2}, {allowed, 4}, {counts, 4}, {token_ids, 4}}))
    return fail(MF_INVALID_ARGUMENT);
  if (hidden_size > UINT32_MAX) return fail(MF_RESOURCE_LIMIT);
  const bool fast = hidden_size == (uint64_t)kFastHidden && (uintptr_t)hidden % 16 == 0 &&
                    (uintptr_t)embedding % 16 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Long tables: a cluster of C CTAs per row, C = 512 ids per CTA rounded up
  // to a power of two, at most 8 (portable cluster size); grid = rows x C.
  uint32_t c = 1;
  while (c < 8 && (uint64_t)c * 512 < max_allowed) c *= 2;
  if (c > 1 && (uint64_t)rows * c > (uint64_t)INT32_MAX) c = 1;
  if (c == 1) {
    auto args = [&](auto kernel) {
      kernel<<<(unsigned)rows, kRowThreads, 0, s>>>(
          static_cast<const __half*>(hidden), static_cast<const __half*>(embedding),
          static_cast<const uint32_t*>(allowed), static_cast<const uint32_t*>(counts),
          static_cast<uint32_t*>(token_ids), (uint32_t)hidden_size, (uint32_t)vocab, max_allowed);
    };
    if (fast)
      args(padded_head_kernel<true>);
    else
      args(padded_head_kernel<false>);
    return launch_status(cudaGetLastError());
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * c), 1, 1);
  cfg.blockDim = dim3(kRowThreads, 1, 1);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = c;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const __half* hp = static_cast<const __half*>(hidden);
  const __half* ep = static_cast<const __half*>(embedding);
  const uint32_t* ap = static_cast<const uint32_t*>(allowed);
  const uint32_t* cp = static_cast<const uint32_t*>(counts);
  uint32_t* op = static_cast<uint32_t*>(token_ids);
  cudaError_t e = fast ? cudaLaunchKernelEx(&cfg, padded_head_kernel<true, true>, hp, ep, ap, cp,
                                            op, (uint32_t)hidden_size, (uint32_t)vocab, max_allowed)
                       : cudaLaunchKernelEx(&cfg, padded_head_kernel<false, true>, hp, ep, ap, cp,
                                            op, (uint32_t)hidden_size, (uint32_t)vocab, max_allowed);
  if (e == cudaSuccess) e = cudaGetLastError();
  return launch_status(e);
}
