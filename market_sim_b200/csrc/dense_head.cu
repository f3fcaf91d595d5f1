// Dense (full-vocabulary) head: tcgen05 GEMM with the greedy argmax fused
// into the TMEM epilogue; logits are never written to memory.
//
// Replaces the reference's two-pass full head: linear_f16 (cublasGemmEx into
// fp16 logits [rows, V], src/cuda/linear.cu:40-104) followed by
// greedy_select_f16 (src/cuda/greedy.cu:21-59, 237-279).  Here the scores
// stay FP32 and only one packed (score, id) key per row leaves the SM.
//
// Tile = 256 hidden rows (M) x 256 vocabulary rows (N) on a pair of CTAs
// (a 2-CTA cluster, tcgen05 cta_group::2); K = hidden width in 64-element
// (128-byte) chunks.  One CTA per SM, persistent:
//   * pair (m, q) keeps hidden tile m resident in shared memory, 128 rows in
//     each CTA (loaded once by TMA, 128-byte swizzle, K-major), and walks
//     vocabulary tiles n = q, q + Q, q + 2Q, ...; each CTA loads 128 of a
//     tile's 256 embedding rows, so an embedding row crosses L2 -> SM once
//     per 256 hidden rows.  The pairs that share an n sequence run together,
//     so each embedding tile comes from DRAM once and from L2 for the others;
//   * warp 0 (one lane) of each CTA streams its half of the embedding chunks
//     with TMA into a 4-stage ring (no multicast: a plain tiled load of this
//     GPU's memory, completing on the leader CTA's barrier);
//   * warp 1 of both CTAs owns TMEM (512 columns = two 128 x 256 f32
//     accumulators per CTA); one lane of the leader CTA issues
//     tcgen05.mma.cta_group::2.kind::f16 (M = 256, N = 256; 4 per chunk),
//     whose commits arrive on the ring's "empty" and the accumulator's
//     "full" barriers of both CTAs;
//   * warps 2-9 of each CTA drain its accumulator with tcgen05.ld while the next
//     tile accumulates: thread = one hidden row and half of the tile's 256
//     columns; per 64 columns a NaN-ignoring max tree, and only when it beats
//     the running best, a search for the lowest column holding it (columns
//     scanned in increasing id order keep the lowest id on ties; NaN never
//     wins).
// At the end each row's key is merged with atomicMax into the workspace; the
// last CTA out decodes keys to ids/scores and clears the workspace.  The key
// order is the selection rule (see common.cuh), so vocabulary shards on
// several GPUs merge with a plain max-reduction of the keys.
//
// Vocabulary shards on several GPUs (mf_dense_head_sharded_f16): the merge
// is fused into the same kernel.  The last CTA on each rank stores its keys
// into every rank's exchange buffer over NVLink (plain peer stores through
// CUDA IPC mappings), raises its epoch flag there with a system-scope
// release, waits (bounded) for every rank's flag in its own buffer, and
// decodes the maximum.  This replaces a NCCL max all-reduce of the keys and
// the decode launch.  Exchange buffer of one rank (mf_exchange_bytes):
//   u32 epoch (this rank's call counter) at 0, u32 broken at 4,
//   u32 flags[world] at 64 (2 x epoch + failed, of rank q's call),
//   u64 slots[2][world][rows] at 512, parity = epoch & 1, so a rank one call
//   ahead never overwrites keys a slower rank is still reading (a rank cannot
//   get two calls ahead: finishing a call needs every rank's flag for it).
// A flag passes only when it names exactly this call.  A wait that runs out
// (100 ms) or a peer reporting a failed part gives every row the sentinel
// and marks the buffer broken: a peer that arrives late could otherwise
// leave keys of an old call where a later call of the same parity reads, so
// every later call on a broken buffer gives the sentinel too, until the
// caller makes new exchange buffers.
//
// (Measured and rejected: every CTA max-reducing its rows' keys into every
// rank's slot as it finishes, 54 us per step on 2 GPUs, and the last CTA of
// each hidden tile pushing the tile's rows, 44 us, against 38 us for this
// single push by the last CTA: the merge sits at the end of the kernel
// either way, and the extra system-scope fences cost more than they hide.)
//
// Every mbarrier wait is bounded; a wait that runs out sets an abort flag
// and the error word in the workspace, and the CTA drains its in-flight
// copies and MMAs (bounded again) before freeing TMEM and exiting.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstring>
#include <initializer_list>
#include <mutex>

#include "common.cuh"

namespace mfb {
namespace dense {

constexpr int kBM = 128;          // hidden rows per CTA (MMA M = 2 x kBM per pair)
constexpr int kBN = 256;          // vocabulary rows per tile (MMA N)
constexpr int kBNHalf = kBN / 2;  // embedding rows each CTA of the pair loads
constexpr int kBK = 64;           // K elements per chunk (one 128-byte swizzle atom)
constexpr int kMaxKChunks = 9;    // hidden width up to 576
constexpr int kStages = 4;        // embedding chunks in flight
constexpr int kAChunkBytes = kBM * kBK * 2;      // 16 KB
constexpr int kBChunkBytes = kBNHalf * kBK * 2;  // 16 KB per CTA
constexpr int kEpiWarps = 8;      // two per TMEM lane quadrant, each on half the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, MMA, epilogue warps
constexpr uint32_t kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 100ull * 1000 * 1000;  // 100 ms per mbarrier wait
constexpr int kMaxRanks = 8;       // GPUs of one node
constexpr int kXFlags = 64;        // exchange buffer: flags offset
constexpr int kXSlots = 512;       // exchange buffer: slots offset

struct Smem {  // offsets inside the 1024-aligned dynamic shared memory
  static constexpr int a = 0;
  static constexpr int b = kMaxKChunks * kAChunkBytes;             // 147,456
  static constexpr int bars = b + kStages * kBChunkBytes;          // 212,992
  // barriers: a_full, b_full[S], b_empty[S], acc_full[2], acc_empty[2], drain
  static constexpr int n_bars = 2 * kStages + 6;
  static constexpr int tmem_slot = bars + n_bars * 8;
  static constexpr int abort_flag = tmem_slot + 4;
  // u32[kStages + 1]: TMA loads issued per stage, then 1 if the hidden tile was
  static constexpr int issued = abort_flag + 4;
  static constexpr int size = issued + 4 * (kStages + 1);
};
constexpr size_t kSmemBytes = Smem::size + 1024;  // + alignment slack

struct Params {
  uint32_t rows;        // hidden rows (batch)
  uint32_t k_chunks;    // hidden width / 64
  uint32_t vocab_rows;  // rows of this vocabulary shard
  uint32_t vocab_begin; // global id of shard row 0
  uint32_t m_tiles, n_tiles, per_m;  // m_tiles: 256-row hidden tiles (pairs)
  unsigned long long* keys;  // workspace: rows keys
  uint32_t* control;         // workspace: done counter, error word
  unsigned long long* out_keys;
  uint32_t* out_ids;
  float* out_scores;
  uint32_t* error_out;       // optional: receives the error word (self-test)
  uint32_t skip_loads;       // self-test only: the producer issues nothing
  uint32_t world, rank;      // vocabulary shards merged in-kernel when world > 1
  unsigned char* xbuf[kMaxRanks];  // every rank's exchange buffer, as mapped here
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void bar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void bar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (any CTA of the cluster).
__device__ __forceinline__ void bar_arrive_cluster(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}

// All threads of both CTAs of the pair; both CTAs always reach it (every
// wait before it is bounded).
__device__ __forceinline__ void cluster_sync() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase of parity `parity` of `bar`, for at most kWaitLimitNs.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  const uint64_t start = global_ns();
  for (uint32_t i = 0;; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred q;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255u) == 255u && global_ns() - start > kWaitLimitNs) return false;
  }
}

// Tiled load into this CTA's shared memory whose completion is counted on
// `leader_bar`, a shared::cluster address of the leader CTA's barrier
// (cta_group::2 lets the barrier live in the peer CTA).  No multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t leader_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(leader_bar)
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;    // leading byte offset (unused for this layout)
  d |= (uint64_t)(1024u >> 4) << 32;  // stride byte offset
  d |= 1ull << 46;                    // descriptor version
  d |= 2ull << 61;                    // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16: F32 accumulator, F16 A and B, both
// K-major, N = 256, M = 256 (the pair's two 128-row halves).
constexpr uint32_t kIdesc =
    (1u << 4) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)((2 * kBM) >> 4) << 24);

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Arrives (once the MMAs issued so far complete) on the barrier at this
// shared-memory offset in both CTAs of the pair.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"((uint16_t)0x3)
      : "memory");
}

// Same, on this CTA's barrier only.
__device__ __forceinline__ void mma_commit_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 TMEM lanes x 64 consecutive f32 columns -> 64 registers per thread.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
dense_head_kernel(const __grid_constant__ CUtensorMap tm_hidden,
                  const __grid_constant__ CUtensorMap tm_emb, Params p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(sm);
  const uint32_t bar0 = sbase + Smem::bars;
  const uint32_t a_full = bar0;
  auto b_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto b_empty = [&](int s) { return bar0 + 8 * (1 + kStages + s); };
  auto acc_full = [&](int b) { return bar0 + 8 * (1 + 2 * kStages + b); };
  auto acc_empty = [&](int b) { return bar0 + 8 * (3 + 2 * kStages + b); };
  const uint32_t drain = bar0 + 8 * (5 + 2 * kStages);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(sm + Smem::abort_flag);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + Smem::tmem_slot);
  volatile uint32_t* issued = reinterpret_cast<volatile uint32_t*>(sm + Smem::issued);
  __shared__ uint32_t s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t rank;  // 0 = leader (issues the MMAs), 1 = peer
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
  const uint32_t pair = blockIdx.x >> 1;
  const uint32_t m = pair % p.m_tiles;  // 256-row hidden tile
  const uint32_t q = pair / p.m_tiles;  // position in the vocabulary walk
  const uint32_t my_tiles = q < p.n_tiles ? (p.n_tiles - q + p.per_m - 1) / p.per_m : 0;
  const bool leader = rank == 0;
  // Overlapped launches (MF_LAUNCH_OVERLAP_PREVIOUS): the next launch's CTA
  // pairs may take SMs as this launch's retire and run their tiles; every
  // write to the workspace or the outputs waits for the previous launch
  // (pdl_wait before the key merge and at teardown).
  pdl_trigger();

  if (threadIdx.x == 0) {
    bar_init(a_full, 1);
    for (int s = 0; s < kStages; ++s) {
      bar_init(b_full(s), 1);
      bar_init(b_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      bar_init(acc_full(b), 1);
      bar_init(acc_empty(b), 2 * kEpiWarps);  // leader's: one arrival per epilogue warp of the pair
    }
    bar_init(drain, 1);
    *abort_flag = 0u;
    for (int s = 0; s <= kStages; ++s) issued[s] = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // TMEM: 512 columns per CTA, two 256-column accumulators
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_before();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t chunks = p.k_chunks;

  if (warp == 0) {
    // ---- producer: hidden tile once, then the embedding chunks ----
    // Both CTAs load their halves; the copies complete on the leader's
    // barriers, whose expected byte counts (set by the leader) cover both.
    if (lane == 0 && my_tiles > 0 && !p.skip_loads) {
      issued[kStages] = 1u;  // the hidden tile
      if (leader) bar_expect_tx(a_full, 2 * chunks * kAChunkBytes);
      for (uint32_t kc = 0; kc < chunks; ++kc)
        tma_load_2d(sbase + Smem::a + kc * kAChunkBytes, &tm_hidden, (int)(kc * kBK),
                    (int)(m * 2 * kBM + rank * kBM), mapa(a_full, 0));
      uint32_t it = 0;
      for (uint32_t t = 0; t < my_tiles && !*abort_flag; ++t) {
        const uint32_t n = q + t * p.per_m;
        for (uint32_t kc = 0; kc < chunks; ++kc, ++it) {
          const int s = (int)(it % kStages);
          const uint32_t ph = (it / kStages) & 1u;
          if (!bar_wait(b_empty(s), ph ^ 1u)) {
            *abort_flag = 1u;
            break;
          }
          if (leader) bar_expect_tx(b_full(s), 2 * kBChunkBytes);
          tma_load_2d(sbase + Smem::b + s * kBChunkBytes, &tm_emb, (int)(kc * kBK),
                      (int)(n * kBN + rank * kBNHalf), mapa(b_full(s), 0));
          issued[s] = issued[s] + 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer (leader CTA only) ----
    if (lane == 0 && my_tiles > 0 && leader) {
      bool ok = bar_wait(a_full, 0);
      uint32_t it = 0;
      for (uint32_t t = 0; ok && t < my_tiles && !*abort_flag; ++t) {
        const uint32_t buf = t & 1u;
        if (!bar_wait(acc_empty(buf), ((t >> 1) & 1u) ^ 1u)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t d = tmem + buf * kBN;
        for (uint32_t kc = 0; kc < chunks; ++kc, ++it) {
          const int s = (int)(it % kStages);
          if (!bar_wait(b_full(s), (it / kStages) & 1u)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t a_addr = sbase + Smem::a + kc * kAChunkBytes;
          const uint32_t b_addr = sbase + Smem::b + s * kBChunkBytes;
#pragma unroll
          for (int k4 = 0; k4 < kBK / 16; ++k4)  // 16-element K steps inside the atom
            mma_f16(d, sw128_desc(a_addr + 32 * k4), sw128_desc(b_addr + 32 * k4),
                    (kc | (uint32_t)k4) != 0u);
          mma_commit_pair(b_empty(s));  // frees the stage (both CTAs) once read
        }
        if (!ok) break;
        mma_commit_pair(acc_full(buf));
      }
      if (!ok) *abort_flag = 1u;
      // all MMAs issued so far complete before either CTA releases TMEM
      mma_commit_local(drain);
      bar_wait(drain, 0);
    }
  } else {
    // ---- epilogue: warps 2-9; warp w serves TMEM lanes 32 (w % 4) .. +31
    // (one hidden row per thread) and column half (w - 2) / 4 of each tile ----
    const uint32_t quad = (uint32_t)(warp & 3);
    const uint32_t half = (uint32_t)(warp - 2) >> 2;
    const uint32_t row = m * 2 * kBM + rank * kBM + quad * 32 + (uint32_t)lane;
    const uint32_t leader_acc_empty0 = mapa(acc_empty(0), 0);
    const uint32_t leader_acc_empty1 = mapa(acc_empty(1), 0);
    const float qnan = __uint_as_float(0x7FC00000u);
    float best = __uint_as_float(0xFF800000u);  // -inf
    uint32_t best_col = 0xFFFFFFFFu;
    for (uint32_t t = 0; t < my_tiles; ++t) {
      const uint32_t buf = t & 1u;
      if (*abort_flag || !bar_wait(acc_full(buf), (t >> 1) & 1u)) {
        *abort_flag = 1u;
        break;
      }
      fence_after();
      const uint32_t n = q + t * p.per_m;
#pragma unroll 1
      for (uint32_t c = 0; c < kBN / 2; c += 64) {
        const uint32_t col0 = n * kBN + half * (kBN / 2) + c;
        uint32_t r[64];
        tmem_ld64(tmem + ((quad * 32u) << 16) + buf * kBN + half * (kBN / 2) + c, r);
        if (col0 + 64 > p.vocab_rows) {  // partial last tile: columns past the shard never win
#pragma unroll
          for (int j = 0; j < 64; ++j)
            if (col0 + j >= p.vocab_rows) r[j] = __float_as_uint(qnan);
        }
        // fmaxf ignores NaN, so mx is the chunk's best real score (NaN only
        // if every score is NaN)
        float mx = __uint_as_float(r[0]);
#pragma unroll
        for (int j = 1; j < 64; ++j) mx = fmaxf(mx, __uint_as_float(r[j]));
        if (mx > best || (best_col == 0xFFFFFFFFu && mx == mx)) {
          int first = 0;  // lowest column holding mx
#pragma unroll
          for (int j = 63; j >= 0; --j) first = __uint_as_float(r[j]) == mx ? j : first;
          best = mx;
          best_col = col0 + (uint32_t)first;
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) bar_arrive_cluster(buf ? leader_acc_empty1 : leader_acc_empty0);
    }
    if (my_tiles > 0 && row < p.rows && !*abort_flag) {
      // all-NaN (or empty) rows: NaN key of the shard's first id, which the
      // key order ranks below every real score and lowest-id first
      const unsigned long long key =
          best_col != 0xFFFFFFFFu ? make_key(best, p.vocab_begin + best_col)
                                  : make_key(qnan, p.vocab_begin);
      pdl_wait();
      atomicMax(p.keys + row, key);
    }
  }

  // ---- teardown: drain the producers' copies, free TMEM ----
  pdl_wait();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    atomicOr(p.control + 1, 1u);
    if (leader) {
      // wait (bounded) for the last copy issued into each stage, and the hidden tile
      for (int s = 0; s < kStages; ++s)
        if (issued[s] > 0u) bar_wait(b_full(s), (issued[s] - 1u) & 1u);
      if (issued[kStages]) bar_wait(a_full, 0);
    } else if (issued[kStages]) {
      // the peer's copies complete on the leader's barriers: give any still
      // in flight 1 ms (a copy of this GPU's memory takes microseconds)
      const uint64_t t0 = global_ns();
      while (global_ns() - t0 < 1000000ull) __nanosleep(10000);
    }
  }
  fence_before();
  cluster_sync();  // no CTA frees TMEM or exits while its pair may still touch it
  fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");

  // ---- last CTA out: decode the merged keys, clear the workspace ----
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(p.control, 1u) == gridDim.x - 1) ? 1u : 0u;
  __syncthreads();
  if (s_last) {
    __threadfence();
    const bool failed = atomicAdd(p.control + 1, 0u) != 0u;
    if (p.world > 1) {
      // ---- fused vocabulary-shard merge over the exchange buffers ----
      __shared__ uint32_t s_epoch, s_xfail;
      unsigned char* self = p.xbuf[p.rank];
      if (threadIdx.x == 0) {
        s_epoch = *reinterpret_cast<volatile uint32_t*>(self) + 1u;
        s_xfail = (failed || *reinterpret_cast<volatile uint32_t*>(self + 4) != 0u) ? 1u : 0u;
      }
      __syncthreads();
      const uint32_t epoch = s_epoch;
      const uint32_t want = epoch & 0x7FFFFFFFu;
      const bool own_fail = s_xfail != 0u;
      const size_t par_off = kXSlots + (size_t)(epoch & 1u) * p.world * p.rows * 8;
      // every CTA's merge is complete and visible (done counter + fences):
      // plain L2 loads, four rows per thread in flight, then the clears
      for (uint32_t r0 = threadIdx.x; r0 < p.rows; r0 += 4 * kThreads) {
        unsigned long long k[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t r = r0 + j * kThreads;
          k[j] = (r < p.rows && !failed) ? __ldcg(p.keys + r) : kKeyPoison;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t r = r0 + j * kThreads;
          if (r >= p.rows) break;
          p.keys[r] = 0ull;
          for (uint32_t q = 0; q < p.world; ++q)
            reinterpret_cast<unsigned long long*>(p.xbuf[q] + par_off)[(size_t)p.rank * p.rows + r] =
                k[j];
        }
      }
      // the block barrier orders every thread's peer stores before the flag
      // writers' system-scope fence and release (one fence per flag, not
      // one per thread)
      __syncthreads();
      if (threadIdx.x < p.world) {  // this rank's flag for this call, in every buffer
        __threadfence_system();
        uint32_t* flag = reinterpret_cast<uint32_t*>(p.xbuf[threadIdx.x] + kXFlags) + p.rank;
        const uint32_t v = (want << 1) | (own_fail ? 1u : 0u);
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
      }
      if (threadIdx.x < p.world && threadIdx.x != p.rank) {
        // wait (bounded) until rank threadIdx.x has stored this call's keys
        // here: the flag must name exactly this call
        const uint32_t* flag = reinterpret_cast<const uint32_t*>(self + kXFlags) + threadIdx.x;
        const uint64_t start = global_ns();
        for (uint32_t i = 0;; ++i) {
          uint32_t v;
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
          if ((v >> 1) == want) {
            if (v & 1u) atomicOr(&s_xfail, 1u);  // that rank failed its part
            break;
          }
          if ((i & 63u) == 63u && global_ns() - start > kWaitLimitNs) {
            atomicOr(&s_xfail, 1u);
            break;
          }
        }
      }
      __syncthreads();
      const bool xfail = s_xfail != 0u;
      if (threadIdx.x == 0 && p.error_out) *p.error_out = xfail ? 1u : 0u;
      const unsigned long long* slots =
          reinterpret_cast<const unsigned long long*>(self + par_off);
      // ordered after the flags' acquire loads by the barrier above; L2
      // loads (not L1: a slot parity is reused every other call), all of a
      // row's slots in flight at once
      for (uint32_t r = threadIdx.x; r < p.rows; r += kThreads) {
        unsigned long long key = 0ull;
#pragma unroll 8
        for (uint32_t q = 0; q < p.world; ++q) key = umax64(key, __ldcg(slots + (size_t)q * p.rows + r));
        if (xfail) key = kKeyPoison;
        if (p.out_keys) p.out_keys[r] = key;
        if (p.out_ids) p.out_ids[r] = key_is_result(key) ? key_id(key) : kInvalid;
        if (p.out_scores)
          p.out_scores[r] = key_is_result(key) ? key_score(key) : __uint_as_float(0x7FC00000u);
      }
      if (threadIdx.x == 0) {
        if (xfail) *reinterpret_cast<volatile uint32_t*>(self + 4) = 1u;  // broken from now on
        *reinterpret_cast<volatile uint32_t*>(self) = epoch;
      }
    } else {
      if (threadIdx.x == 0 && p.error_out) *p.error_out = failed ? 1u : 0u;
      for (uint32_t r0 = threadIdx.x; r0 < p.rows; r0 += 4 * kThreads) {
        unsigned long long k[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t r = r0 + j * kThreads;
          k[j] = (r < p.rows && !failed) ? __ldcg(p.keys + r) : kKeyPoison;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t r = r0 + j * kThreads;
          if (r >= p.rows) break;
          p.keys[r] = 0ull;
          const unsigned long long key = k[j];
          if (p.out_keys) p.out_keys[r] = key;
          if (p.out_ids) p.out_ids[r] = key_is_result(key) ? key_id(key) : kInvalid;
          if (p.out_scores)
            p.out_scores[r] = key_is_result(key) ? key_score(key) : __uint_as_float(0x7FC00000u);
        }
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      p.control[1] = 0u;
      p.control[0] = 0u;
    }
  }
}

// Decodes merged keys (after a cross-GPU max-reduction) to ids and scores.
__global__ void decode_keys_kernel(const unsigned long long* keys, uint32_t rows, uint32_t* ids,
                                   float* scores) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const unsigned long long key = keys[r];
  if (ids) ids[r] = key_is_result(key) ? key_id(key) : kInvalid;
  if (scores) scores[r] = key_is_result(key) ? key_score(key) : __uint_as_float(0x7FC00000u);
}

}  // namespace dense
}  // namespace mfb

using namespace mfb;
using namespace mfb::dense;

namespace {

mf_status d_ok() { return mf_status{MF_OK, 0}; }
mf_status d_fail(int32_t code, uint32_t detail = 0) { return mf_status{code, detail}; }

bool d_distinct(std::initializer_list<const void*> ptrs) {
  const void* seen[16];
  int n = 0;
  for (const void* q : ptrs) {
    if (q == nullptr) continue;
    for (int i = 0; i < n; ++i)
      if (seen[i] == q) return false;
    seen[n++] = q;
  }
  return true;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// 2-D tensor map over fp16 [rows, width] with (64 x box_rows) boxes, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t width,
              uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {width, rows};
  const cuuint64_t strides[1] = {width * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Sets the kernel's shared-memory limit (once per device) and returns how
// many CTA pairs can be resident at once: at most SMs / 2, fewer where a GPC
// has an odd number of SMs free, so that the persistent grid is one wave.
cudaError_t resident_pairs(int dev, int sms, uint32_t* pairs) {
  static std::mutex mu;
  static int cached[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  int& c = cached[dev & 63];
  if (c == 0) {
    cudaError_t e = cudaFuncSetAttribute(
        dense_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(sms & ~1), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, dense_head_kernel, &cfg);
    if (e != cudaSuccess) return e;
    c = clusters < 1 ? 1 : (clusters > sms / 2 ? sms / 2 : clusters);
  }
  *pairs = (uint32_t)c;
  return cudaSuccess;
}

}  // namespace

extern "C" uint64_t mf_dense_workspace_bytes(uint64_t rows) { return ((rows * 8 + 16) + 15) & ~15ull; }

namespace {

// Validates and launches the dense head; world > 1 merges the vocabulary
// shards in-kernel through the exchange buffers `xbuf` (already checked).
mf_status dense_launch(const void* hidden, uint64_t hidden_bytes, const void* embedding,
                       uint64_t embedding_bytes, void* out_keys, uint64_t out_keys_bytes,
                       void* out_ids, uint64_t out_ids_bytes, void* out_scores,
                       uint64_t out_scores_bytes, void* workspace, uint64_t workspace_bytes,
                       uint64_t rows, uint64_t hidden_size, uint64_t vocab_rows,
                       uint64_t vocab_begin, uint32_t world, uint32_t rank,
                       unsigned char* const* xbuf, uint32_t launch_flags, void* stream) {
  if (rows == 0 || hidden_size == 0 || vocab_rows == 0 || stream == nullptr ||
      (launch_flags & ~MF_LAUNCH_OVERLAP_PREVIOUS) != 0)
    return d_fail(MF_INVALID_ARGUMENT);
  if (hidden_size % kBK != 0 || hidden_size > (uint64_t)kMaxKChunks * kBK)
    return d_fail(MF_RESOURCE_LIMIT);  // widths 64..576 in steps of 64
  if (vocab_rows > UINT32_MAX || vocab_begin + vocab_rows > UINT32_MAX ||
      rows > (uint64_t)INT32_MAX)
    return d_fail(MF_RESOURCE_LIMIT);
  if (hidden_bytes != rows * hidden_size * 2 || embedding_bytes != vocab_rows * hidden_size * 2 ||
      (out_keys && out_keys_bytes != rows * 8) || (out_ids && out_ids_bytes != rows * 4) ||
      (out_scores && out_scores_bytes != rows * 4) ||
      workspace_bytes < mf_dense_workspace_bytes(rows) || hidden == nullptr ||
      embedding == nullptr || workspace == nullptr ||
      (out_keys == nullptr && out_ids == nullptr) ||
      !d_distinct({hidden, embedding, out_keys, out_ids, out_scores, workspace}) ||
      (uintptr_t)hidden % 16 != 0 || (uintptr_t)embedding % 16 != 0 ||
      (uintptr_t)out_keys % 8 != 0 || (uintptr_t)out_ids % 4 != 0 ||
      (uintptr_t)out_scores % 4 != 0 || (uintptr_t)workspace % 8 != 0)
    return d_fail(MF_INVALID_ARGUMENT);
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
  Params p{};
  p.rows = (uint32_t)rows;
  p.k_chunks = (uint32_t)(hidden_size / kBK);
  p.vocab_rows = (uint32_t)vocab_rows;
  p.vocab_begin = (uint32_t)vocab_begin;
  p.m_tiles = (uint32_t)((rows + 2 * kBM - 1) / (2 * kBM));
  p.n_tiles = (uint32_t)((vocab_rows + kBN - 1) / kBN);
  uint32_t pairs = 0;
  e = resident_pairs(dev, sms, &pairs);
  if (e != cudaSuccess) return d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
  if (p.m_tiles > pairs) return d_fail(MF_RESOURCE_LIMIT);  // rows <= 256 x SM pairs
  p.per_m = pairs / p.m_tiles;
  if (p.per_m > p.n_tiles) p.per_m = p.n_tiles;
  char* ws = static_cast<char*>(workspace);
  p.keys = reinterpret_cast<unsigned long long*>(ws);
  p.control = reinterpret_cast<uint32_t*>(ws + rows * 8);
  p.out_keys = static_cast<unsigned long long*>(out_keys);
  p.out_ids = static_cast<uint32_t*>(out_ids);
  p.out_scores = static_cast<float*>(out_scores);
  p.world = world;
  p.rank = rank;
  if (world > 1)  // the caller checked world <= kMaxRanks and every pointer
    for (uint32_t q = 0; q < world; ++q) p.xbuf[q] = xbuf[q];
  CUtensorMap tm_h, tm_e;
  if (!make_map(&tm_h, hidden, rows, hidden_size, kBM) ||
      !make_map(&tm_e, embedding, vocab_rows, hidden_size, kBNHalf))
    return d_fail(MF_CUDA_RUNTIME_FAILURE);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * p.m_tiles * p.per_m, 1, 1);  // CTA pairs (cluster dims 2)
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  if (launch_flags & MF_LAUNCH_OVERLAP_PREVIOUS) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  e = cudaLaunchKernelEx(&cfg, dense_head_kernel, tm_h, tm_e, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  return e == cudaSuccess ? d_ok() : d_fail(MF_CUDA_BACKEND_FAILURE, (uint32_t)e);
}

}  // namespace

extern "C" mf_status mf_dense_head_f16(const void* hidden, uint64_t hidden_bytes,
                                       const void* embedding, uint64_t embedding_bytes,
                                       void* out_keys, uint64_t out_keys_bytes, void* out_ids,
                                       uint64_t out_ids_bytes, void* out_scores,
                                       uint64_t out_scores_bytes, void* workspace,
                                       uint64_t workspace_bytes, uint64_t rows,
                                       uint64_t hidden_size, uint64_t vocab_rows,
                                       uint64_t vocab_begin, void* stream) {
  return dense_launch(hidden, hidden_bytes, embedding, embedding_bytes, out_keys,
                      out_keys_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes,
                      workspace, workspace_bytes, rows, hidden_size, vocab_rows, vocab_begin, 1u,
                      0u, nullptr, 0u, stream);
}

extern "C" mf_status mf_dense_head_f16_ex(const void* hidden, uint64_t hidden_bytes,
                                          const void* embedding, uint64_t embedding_bytes,
                                          void* out_keys, uint64_t out_keys_bytes, void* out_ids,
                                          uint64_t out_ids_bytes, void* out_scores,
                                          uint64_t out_scores_bytes, void* workspace,
                                          uint64_t workspace_bytes, uint64_t rows,
                                          uint64_t hidden_size, uint64_t vocab_rows,
                                          uint64_t vocab_begin, uint32_t launch_flags,
                                          void* stream) {
  return dense_launch(hidden, hidden_bytes, embedding, embedding_bytes, out_keys,
                      out_keys_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes,
                      workspace, workspace_bytes, rows, hidden_size, vocab_rows, vocab_begin, 1u,
                      0u, nullptr, launch_flags, stream);
}

extern "C" uint64_t mf_exchange_bytes(uint64_t rows, uint32_t world) {
  return (uint64_t)kXSlots + 2ull * world * rows * 8ull;
}

extern "C" mf_status mf_exchange_alloc(void** buffer, uint64_t bytes, void* ipc_handle) {
  if (buffer == nullptr || ipc_handle == nullptr || bytes < (uint64_t)kXSlots)
    return d_fail(MF_INVALID_ARGUMENT);
  *buffer = nullptr;
  void* b = nullptr;
  cudaError_t e = cudaMalloc(&b, bytes);
  if (e == cudaSuccess) e = cudaMemset(b, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, b);
  if (e != cudaSuccess) {
    cudaFree(b);
    return d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
  }
  static_assert(sizeof(h) == MF_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *buffer = b;
  return d_ok();
}

extern "C" mf_status mf_exchange_free(void* buffer) {
  const cudaError_t e = cudaFree(buffer);
  return e == cudaSuccess ? d_ok() : d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
}

extern "C" mf_status mf_exchange_open_peer(const void* ipc_handle, void** peer_buffer) {
  if (ipc_handle == nullptr || peer_buffer == nullptr) return d_fail(MF_INVALID_ARGUMENT);
  *peer_buffer = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? d_ok() : d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
}

extern "C" mf_status mf_exchange_broken(const void* buffer, uint32_t* broken) {
  if (buffer == nullptr || broken == nullptr) return d_fail(MF_INVALID_ARGUMENT);
  const cudaError_t e = cudaMemcpy(broken, static_cast<const char*>(buffer) + 4, 4,
                                   cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? d_ok() : d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
}

extern "C" mf_status mf_exchange_close_peer(void* peer_buffer) {
  const cudaError_t e = cudaIpcCloseMemHandle(peer_buffer);
  return e == cudaSuccess ? d_ok() : d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
}

extern "C" mf_status mf_dense_head_sharded_f16(
    const void* hidden, uint64_t hidden_bytes, const void* embedding, uint64_t embedding_bytes,
    void* out_keys, uint64_t out_keys_bytes, void* out_ids, uint64_t out_ids_bytes,
    void* out_scores, uint64_t out_scores_bytes, void* workspace, uint64_t workspace_bytes,
    uint64_t rows, uint64_t hidden_size, uint64_t vocab_rows, uint64_t vocab_begin,
    void* const* exchange, uint64_t exchange_bytes, uint32_t world, uint32_t rank,
    uint32_t launch_flags, void* stream) {
  if (world == 0 || rank >= world || exchange == nullptr) return d_fail(MF_INVALID_ARGUMENT);
  if (world > (uint32_t)kMaxRanks) return d_fail(MF_RESOURCE_LIMIT);
  if (exchange_bytes < mf_exchange_bytes(rows, world)) return d_fail(MF_INVALID_ARGUMENT);
  unsigned char* xbuf[kMaxRanks] = {};
  for (uint32_t q = 0; q < world; ++q) {
    xbuf[q] = static_cast<unsigned char*>(exchange[q]);
    if (xbuf[q] == nullptr || (uintptr_t)xbuf[q] % 256 != 0) return d_fail(MF_INVALID_ARGUMENT);
    for (uint32_t j = 0; j < q; ++j)
      if (xbuf[j] == xbuf[q]) return d_fail(MF_INVALID_ARGUMENT);
  }
  return dense_launch(hidden, hidden_bytes, embedding, embedding_bytes, out_keys,
                      out_keys_bytes, out_ids, out_ids_bytes, out_scores, out_scores_bytes,
                      workspace, workspace_bytes, rows, hidden_size, vocab_rows, vocab_begin,
                      world, rank, xbuf, launch_flags, stream);
}

extern "C" mf_status mf_decode_keys(const void* keys, uint64_t keys_bytes, void* out_ids,
                                    uint64_t out_ids_bytes, void* out_scores,
                                    uint64_t out_scores_bytes, uint64_t rows, void* stream) {
  if (rows == 0 || stream == nullptr || keys == nullptr || out_ids == nullptr)
    return d_fail(MF_INVALID_ARGUMENT);
  if (rows > (uint64_t)INT32_MAX) return d_fail(MF_RESOURCE_LIMIT);
  if (keys_bytes != rows * 8 || out_ids_bytes != rows * 4 ||
      (out_scores && out_scores_bytes != rows * 4) || !d_distinct({keys, out_ids, out_scores}) ||
      (uintptr_t)keys % 8 != 0 || (uintptr_t)out_ids % 4 != 0 || (uintptr_t)out_scores % 4 != 0)
    return d_fail(MF_INVALID_ARGUMENT);
  decode_keys_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned long long*>(keys), (uint32_t)rows, static_cast<uint32_t*>(out_ids),
      static_cast<float*>(out_scores));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? d_ok() : d_fail(MF_CUDA_BACKEND_FAILURE, (uint32_t)e);
}

// Self-test of the bounded waits (no counterpart in the reference): runs a
// 128 x 256 x 64 dense problem (one CTA pair) whose producers issue no loads, so the MMA
// and epilogue waits run out (100 ms each).  The kernel must return, give
// every row the sentinel and report the error word; the context stays
// usable.  Allocates its small buffers with cudaMalloc and synchronises.
extern "C" mf_status mf_dense_selftest_wait_timeout(void* stream, uint32_t* error_word,
                                                    uint32_t* invalid_rows) {
  if (stream == nullptr || error_word == nullptr || invalid_rows == nullptr)
    return d_fail(MF_INVALID_ARGUMENT);
  const uint64_t rows = 128, hs = 64, vocab = 256;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void *hid = nullptr, *emb = nullptr, *ws = nullptr, *ids = nullptr, *err = nullptr;
  cudaError_t e = cudaMalloc(&hid, rows * hs * 2);
  if (e == cudaSuccess) e = cudaMalloc(&emb, vocab * hs * 2);
  if (e == cudaSuccess) e = cudaMalloc(&ws, mf_dense_workspace_bytes(rows));
  if (e == cudaSuccess) e = cudaMalloc(&ids, rows * 4);
  if (e == cudaSuccess) e = cudaMalloc(&err, 4);
  if (e == cudaSuccess) e = cudaMemsetAsync(hid, 0, rows * hs * 2, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(emb, 0, vocab * hs * 2, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(ws, 0, mf_dense_workspace_bytes(rows), s);
  mf_status st = d_ok();
  int dev = 0, sms = 0;
  if (e == cudaSuccess) e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  CUtensorMap tm_h, tm_e;
  if (e == cudaSuccess &&
      (!make_map(&tm_h, hid, rows, hs, kBM) || !make_map(&tm_e, emb, vocab, hs, kBNHalf)))
    st = d_fail(MF_CUDA_RUNTIME_FAILURE);
  uint32_t pairs = 0;
  if (e == cudaSuccess && st.code == MF_OK) e = resident_pairs(dev, sms, &pairs);
  if (e == cudaSuccess && st.code == MF_OK) {
    Params p{};
    p.rows = (uint32_t)rows;
    p.k_chunks = 1;
    p.vocab_rows = (uint32_t)vocab;
    p.m_tiles = 1;
    p.n_tiles = 1;
    p.per_m = 1;
    p.keys = static_cast<unsigned long long*>(ws);
    p.control = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + rows * 8);
    p.out_ids = static_cast<uint32_t*>(ids);
    p.error_out = static_cast<uint32_t*>(err);
    p.skip_loads = 1u;
    dense_head_kernel<<<2, kThreads, kSmemBytes, s>>>(tm_h, tm_e, p);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  if (e == cudaSuccess && st.code == MF_OK) {
    uint32_t host_ids[128];
    e = cudaMemcpy(host_ids, ids, sizeof(host_ids), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(error_word, err, 4, cudaMemcpyDeviceToHost);
    uint32_t bad = 0;
    for (uint32_t id : host_ids) bad += id == kInvalid;
    *invalid_rows = bad;
  }
  cudaFree(hid);
  cudaFree(emb);
  cudaFree(ws);
  cudaFree(ids);
  cudaFree(err);
  if (st.code != MF_OK) return st;
  return e == cudaSuccess ? d_ok() : d_fail(MF_CUDA_RUNTIME_FAILURE, (uint32_t)e);
}
