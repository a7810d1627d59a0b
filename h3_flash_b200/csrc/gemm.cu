// Bf16 GEMM for B200 (sm_100a), y = x W^T (+ b), with the epilogue fused into
// the kernel. Four epilogues share one pipeline:
//
//   QkvEpi     the QKV projection followed by the packed-Ulysses QK-norm + RoPE +
//              pack: q, k head rows get RMSNorm over D (fp32, eps, weight) and
//              rotate-half RoPE on the first ROT columns, v rows pass; each head
//              row goes to its owner: the destination-major send buffer
//              [W, rows, hl, 3D] (one GPU, or an NCCL all-to-all after), or every
//              owner's receive buffer [S_total, hl, 3D] at its global row over
//              NVLink (p2p). Replaces to_q/to_k/to_v and fused_qknorm_rope + pack
//              of src/h3_flash/runtime/parallel/packed_ulysses.py:166-199
//              (relayout.py:97-130, kernels/fusions.py:125-175).
//   DenseEpi   bias, then nothing or GELU-tanh (the FFN projection of
//              src/h3_flash/runtime/kernels/transformer.py:121-122 with its
//              activation), row-major output.
//   SwigluEpi  W's rows interleaved by 128 (value block b, then gate block b), so
//              each 256-column tile holds matching value and gate columns; the
//              output is value * silu(gate), 128 columns per tile (the SwiGLU
//              projection and fused_swiglu of transformer.py:112-120,
//              fusions.py:251-265).
//
// Tiles are 256 x 256 output elements per CTA pair (tcgen05.mma.cta_group::2,
// M = 256, N = 256, K = 16): CTA c of the pair loads rows [128c, 128c+128) of
// the x tile and rows [128c, 128c+128) of the W tile (output columns) into
// its own shared memory, one leader thread issues the MMAs for both SMs, and
// each CTA's TMEM receives the accumulator of its own 128 rows (all 256
// columns).
//
// Warp roles per CTA (192 threads):
//   warp 0      TMA producer: x and W K-blocks of 64 into a 6-stage ring
//               (32 KB per stage), completion counted on the leader's barrier.
//   warp 1      TMEM allocator (both CTAs) and, in the leader, the MMA issuer.
//   warps 2-5   epilogue: warp w reads TMEM lane quadrant w % 4, one row per
//               thread, in 128-column segments; two 256-column fp32
//               accumulators in TMEM let the epilogue of tile i overlap the MMAs
//               of tile i + 1. A thread writes its row's segment (256 bytes of
//               bf16) into its warp's 8 KB staging buffer; the warp then stores
//               two whole 256-byte rows per instruction (16 bytes per lane), so
//               every output row, local or a peer's over NVLink, is written in
//               full 32-byte sectors.
// The kernel is persistent: pair p of P processes tiles p, p + P, ... in
// row-major tile order (consecutive tiles share the x rows, W stays in L2).
//
// Every mbarrier wait is bounded (2 s). On expiry the thread ORs status bit 4
// into the library status word, raises the CTA's abort flag and unwinds; after
// an abort every thread waits 200 us (TMA copies in flight land) before the
// pair meets at the final cluster barrier and frees TMEM.
//
// No TMA load uses multicast: each CTA loads only into its own shared memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace h3b {
namespace gemm {

constexpr int kBM = 128;        // x rows per CTA (256 per pair)
constexpr int kBN = 256;        // output columns per tile (two heads of the QKV projection)
constexpr int kBNc = kBN / 2;   // W rows each CTA loads
constexpr int kBK = 64;         // K per stage: one 128-byte swizzle row
// Shared-memory ring depth (32 KB per stage); a build-time knob for tuning.
#ifndef H3B_GEMM_STAGES
#define H3B_GEMM_STAGES 6
#endif
constexpr int kStages = H3B_GEMM_STAGES;
constexpr int kEpiWarps = 4;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kHeadDim = 128;
constexpr uint32_t kABytes = kBM * kBK * 2;   // 16 KB
constexpr uint32_t kBBytes = kBNc * kBK * 2;  // 16 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
// Epilogue staging: per epilogue warp, 32 rows x 256 bytes (one 128-column bf16
// segment per row), its 16-byte chunks XOR-swizzled by row so that both the
// per-thread row writes and the per-warp row reads are free of bank conflicts.
constexpr uint32_t kSegBytes = 256;
constexpr uint32_t kEpiStageBytes = 32 * kSegBytes;  // 8 KB
constexpr uint32_t kSmemEpi = kStages * kStageBytes;
constexpr uint32_t kSmemBar = kSmemEpi + kEpiWarps * kEpiStageBytes;
constexpr uint32_t kNumBars = 2 * kStages + 4;  // full[S], empty[S], tfull[2], tempty[2]
constexpr uint32_t kSmemBytes = kSmemBar + kNumBars * 8 + 16;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;  // slack to 1024-align the base
static_assert(kSmemAlloc <= 232448, "shared memory per CTA");
constexpr uint32_t kTmemCols = 512;  // two 256-column fp32 accumulators
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
constexpr unsigned long long kDrainNs = 200000ull;
constexpr unsigned int kStatusGemmTimeout = 4u;

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both operands K-major,
// M = 256 (the pair), N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) |
                            ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)((2 * kBM) >> 4) << 24);

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of the same shared-memory offset in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity (arrivals may come from the
// other CTA of the pair). False if the CTA aborted or this wait timed out.
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity,
                                         volatile uint32_t* abort_flag, unsigned int* status) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        *abort_flag = 1u;
        if (status) atomicOr(status, kStatusGemmTimeout);
        return false;
      }
    }
  }
}

// 2-D TMA load into this CTA's shared memory, completion counted on the
// leader CTA's barrier (`bar` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

// 2-D TMA store of a shared-memory box to global memory (bulk-group completion). The
// output lines are marked evict-first in L2, so that the x and W panels the following
// tiles re-read stay resident (FFN projection: 2.26 GB of DRAM reads per launch with the
// default policy, and faster with the hint in a same-process A/B).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], "
      "%4;" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// This thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// This thread's bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Generic-proxy shared-memory writes become visible to the async proxy (TMA).
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor, 128B swizzle, sm_100 version field.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}

// Completion of this thread's earlier MMAs, arrived on `bar` in both CTAs.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], m;\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// After tcgen05.wait::ld: ties each loaded register to this point of the program, so
// no use of it can be scheduled above the wait.
template <int N>
__device__ __forceinline__ void pin(uint32_t (&r)[N]) {
#pragma unroll
  for (int j = 0; j < N; ++j) asm volatile("" : "+r"(r[j]));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// QKV destinations (the layouts of h3b_qknorm_rope_pack and h3b_qknorm_rope_pack_p2p)
// ---------------------------------------------------------------------------

struct LocalSend {
  static constexpr bool kStaged = false;  // local HBM: L2 merges the row pieces
  __nv_bfloat16* send;  // [W, rows, hl, 3D]
  int64_t rows;
  int hl;
  __device__ __forceinline__ __nv_bfloat16* at(int64_t row, int g, int part) const {
    const int dst = g / hl, lh = g - dst * hl;
    return send + (((int64_t)dst * rows + row) * hl + lh) * (3 * kHeadDim) + part * kHeadDim;
  }
  __device__ __forceinline__ void finish() const {}
};

struct PeerRecv {
  static constexpr bool kStaged = true;  // NVLink: write whole 256-byte rows
  PeerPtrs recv;  // every rank's [S_total, hl, 3D], this rank's own included
  int64_t row_offset;
  int hl;
  __device__ __forceinline__ __nv_bfloat16* at(int64_t row, int g, int part) const {
    const int dst = g / hl, lh = g - dst * hl;
    return reinterpret_cast<__nv_bfloat16*>(peer_at(recv, dst)) +
           ((row_offset + row) * hl + lh) * (3 * kHeadDim) + part * kHeadDim;
  }
  // Peers read these rows after a cross-rank barrier; order the stores first.
  __device__ __forceinline__ void finish() const { __threadfence_system(); }
};

// Shape and status shared by every epilogue.
struct Shape {
  int64_t rows;          // x rows
  int dim;               // K, a multiple of 64
  int tiles_m, tiles_n;  // tiles of 256 rows, 256 columns
  int group_n;           // tile columns per raster group (see tile_coords)
  unsigned int* status;
};

// Tile order. Tiles go in groups of `group_n` tile columns; inside a group the
// columns vary fastest, then the 256-row blocks. The pairs working at one time
// then share one panel of W (group_n x 256 rows of it, sized by the host to stay
// in L2) and a few blocks of x, and each W panel is read from DRAM about once
// instead of once per row block.
__device__ __forceinline__ void tile_coords(int tile, const Shape& s, int& tm, int& tn) {
  const int per_group = s.tiles_m * s.group_n;
  const int g = tile / per_group;
  const int r = tile - g * per_group;
  const int width = min(s.group_n, s.tiles_n - g * s.group_n);
  tm = r / width;
  tn = g * s.group_n + (r - tm * width);
}

// ---------------------------------------------------------------------------
// Epilogues. Each one turns a thread's row of a 256-column fp32 accumulator into
// kSegments segments of 128 bf16 output values, written by ``fill`` into the
// thread's staging row (put8(chunk, 8 floats) stores one 16-byte chunk), and
// names each segment's 256-byte destination with ``dest``.
// ---------------------------------------------------------------------------

// Loads 32 accumulator columns of this thread's row as floats.
__device__ __forceinline__ void load32(uint32_t taddr, float (&x)[32]) {
  uint32_t v[32];
  tmem_ld32(taddr, v);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(v[j]);
}

// QKV projection + QK-norm + RoPE + pack. A 256-column tile never straddles q, k
// and v (H D is a multiple of 256) and holds two heads: segment h is head g0 + h,
// so the RMSNorm sum and every RoPE partner are in the thread's own registers.
template <int ROT, class Dst>
struct QkvEpi {
  static constexpr int kSegments = 2;
  static constexpr bool kStaged = Dst::kStaged;
  static constexpr bool kTmaStore = false;
  static constexpr int kHalf = ROT / 2;
  static_assert(kHalf % 16 == 0, "rotary width: a multiple of 32");
  const __nv_bfloat16* bias;  // [3 H D] or nullptr
  const __nv_bfloat16* wq;    // [D]
  const __nv_bfloat16* wk;    // [D]
  const float4* tab;          // RoPE tables in the epilogue's layout (rope_tables_kernel)
  int64_t tab_rows;
  float q_eps, k_eps;
  int heads;
  Dst dst;

  // bias + accumulator for 8 columns starting at column c of the segment
  __device__ __forceinline__ void biased8(const uint32_t* v, int col, float (&x)[8]) const {
#pragma unroll
    for (int j = 0; j < 8; ++j) x[j] = __uint_as_float(v[j]);
    if (bias != nullptr) {
      const f8 bv = unpack8(ld_cached(bias + col));
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] += bv.v[j];
    }
  }

  // RoPE table slots of rotary chunk k (16 rotate-half pairs) for this thread's row.
  __device__ __forceinline__ void load_tab(int k, int64_t row, float4 (&t)[16]) const {
#pragma unroll
    for (int j = 0; j < 16; ++j) t[j] = __ldg(tab + (int64_t)(16 * k + j) * tab_rows + row);
  }

  // One head row (128 accumulator columns) per call, in two passes so that the row
  // never sits in registers whole: pass 1 sums the squares of the biased projection;
  // pass 2 re-reads it, 16 rotate-half pairs at a time, normalises and rotates them.
  // The RoPE tables come from a row-contiguous layout, so a warp's table load of its
  // 32 consecutive rows is one 512-byte span, and the next chunk's tables are in flight
  // while the current chunk is computed.
  template <class Put>
  __device__ __forceinline__ void fill(uint32_t tacc, int seg, int64_t row, int n0, Put put8) const {
    const int hd = heads * kHeadDim;
    const int col0 = n0 + seg * kHeadDim;
    const int part = col0 / hd;  // 0 q, 1 k, 2 v
    const uint32_t t = tacc + (uint32_t)(seg * kHeadDim);
    float r = 1.f;
    const __nv_bfloat16* w = part == 0 ? wq : wk;
    float4 cur[16];
    if (part < 2) {
      if constexpr (ROT > 0) load_tab(0, row, cur);
      // pass 1: the sum of squares, in column order; the next 32 columns load meanwhile
      float ss = 0.f;
      uint32_t v[2][32];
      tmem_ld32(t, v[0]);
      tmem_ld_wait();
      pin(v[0]);
#pragma unroll
      for (int q4 = 0; q4 < kHeadDim / 32; ++q4) {
        if (q4 + 1 < kHeadDim / 32) tmem_ld32(t + (uint32_t)(32 * (q4 + 1)), v[(q4 + 1) & 1]);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float x[8];
          biased8(v[q4 & 1] + 8 * c8, col0 + 32 * q4 + 8 * c8, x);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += x[j] * x[j];
        }
        if (q4 + 1 < kHeadDim / 32) {
          tmem_ld_wait();
          pin(v[(q4 + 1) & 1]);
        }
      }
      r = rsqrtf(ss / (float)kHeadDim + (part == 0 ? q_eps : k_eps));
    }
    if constexpr (ROT > 0) {
      if (part < 2) {
        // pass 2, rotary columns: pairs (c, c + kHalf) for c in [16k, 16k + 16)
#pragma unroll
        for (int k = 0; k < kHalf / 16; ++k) {
          float4 nxt[16];
          if (k + 1 < kHalf / 16) load_tab(k + 1, row, nxt);
          uint32_t va[16], vb[16];
          tmem_ld16(t + (uint32_t)(16 * k), va);
          tmem_ld16(t + (uint32_t)(kHalf + 16 * k), vb);
          tmem_ld_wait();
          pin(va);
          pin(vb);
          const float* ca = reinterpret_cast<const float*>(cur);       // cos[c]
          const float* sa = reinterpret_cast<const float*>(cur + 4);   // sin[c]
          const float* cb = reinterpret_cast<const float*>(cur + 8);   // cos[c + kHalf]
          const float* sb = reinterpret_cast<const float*>(cur + 12);  // sin[c + kHalf]
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float a[8], b[8];
            biased8(va + 8 * h, col0 + 16 * k + 8 * h, a);
            biased8(vb + 8 * h, col0 + kHalf + 16 * k + 8 * h, b);
            const f8 wa = unpack8(ld_cached(w + 16 * k + 8 * h));
            const f8 wb = unpack8(ld_cached(w + kHalf + 16 * k + 8 * h));
            float oa[8], ob[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float an = a[j] * r * wa.v[j], bn = b[j] * r * wb.v[j];
              const int c = 8 * h + j;
              oa[j] = an * ca[c] + (-bn) * sa[c];  // first half takes -partner
              ob[j] = bn * cb[c] + an * sb[c];
            }
            put8(2 * k + h, oa);
            put8(kHalf / 8 + 2 * k + h, ob);
          }
          if (k + 1 < kHalf / 16) {
#pragma unroll
            for (int j = 0; j < 16; ++j) cur[j] = nxt[j];
          }
        }
      }
    }
    if (part < 2)
      rest<ROT / 32>(t, col0, true, r, w, put8);
    else
      rest<0>(t, col0, false, 1.f, w, put8);
  }

  // Columns [32 kFirst, 128) of the head row: normalised (q, k) or biased only (v),
  // 32 at a time with the next 32 in flight.
  template <int kFirst, class Put>
  __device__ __forceinline__ void rest(uint32_t t, int col0, bool norm, float r,
                                       const __nv_bfloat16* w, Put& put8) const {
    if constexpr (kFirst < kHeadDim / 32) {
      uint32_t v[2][32];
      tmem_ld32(t + (uint32_t)(32 * kFirst), v[kFirst & 1]);
      tmem_ld_wait();
      pin(v[kFirst & 1]);
#pragma unroll
      for (int q4 = kFirst; q4 < kHeadDim / 32; ++q4) {
        if (q4 + 1 < kHeadDim / 32) tmem_ld32(t + (uint32_t)(32 * (q4 + 1)), v[(q4 + 1) & 1]);
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          const int c = 32 * q4 + 8 * c8;
          float x[8];
          biased8(v[q4 & 1] + 8 * c8, col0 + c, x);
          if (norm) {
            const f8 wv = unpack8(ld_cached(w + c));
#pragma unroll
            for (int j = 0; j < 8; ++j) x[j] = x[j] * r * wv.v[j];
          }
          put8(c / 8, x);
        }
        if (q4 + 1 < kHeadDim / 32) {
          tmem_ld_wait();
          pin(v[(q4 + 1) & 1]);
        }
      }
    }
  }

  __device__ __forceinline__ __nv_bfloat16* dest(int seg, int64_t row, int n0) const {
    const int hd = heads * kHeadDim;
    const int part = n0 / hd;
    return dst.at(row, (n0 - part * hd) / kHeadDim + seg, part);
  }
  __device__ __forceinline__ void finish() const { dst.finish(); }
};

enum Activation : int { kActNone = 0, kActGeluTanh = 1 };

// y = act(x W^T + b) into a row-major [rows, N] output.
template <int ACT>
struct DenseEpi {
  static constexpr int kSegments = 2;
  // The segment goes through the staging buffer and leaves as two TMA stores (see the
  // epilogue role); the QKV and gated-residual epilogues measured faster storing each
  // thread's row directly.
  static constexpr bool kStaged = true;
  static constexpr bool kTmaStore = true;
  CUtensorMap out_map;  // out [rows, N], (64, 32) box, 128-byte swizzle
  __nv_bfloat16* out;
  int64_t ldo;
  const __nv_bfloat16* bias;  // [N] or nullptr

  template <class Put>
  __device__ __forceinline__ void fill(uint32_t tacc, int seg, int64_t, int n0, Put put8) const {
#pragma unroll 1
    for (int q4 = 0; q4 < 4; ++q4) {
      float x[32];
      load32(tacc + (uint32_t)(seg * 128 + 32 * q4), x);
      const int col0 = n0 + seg * 128 + 32 * q4;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        if (bias != nullptr) {
          const f8 bv = unpack8(ld_cached(bias + col0 + 8 * c8));
#pragma unroll
          for (int j = 0; j < 8; ++j) x[8 * c8 + j] += bv.v[j];
        }
        if (ACT == kActGeluTanh) {
#pragma unroll
          for (int j = 0; j < 8; ++j) x[8 * c8 + j] = gelu_tanh(x[8 * c8 + j]);
        }
        put8(4 * q4 + c8, x + 8 * c8);
      }
    }
  }
  __device__ __forceinline__ __nv_bfloat16* dest(int seg, int64_t row, int n0) const {
    return out + row * ldo + n0 + seg * 128;
  }
  __device__ __forceinline__ void finish() const {}
};

// out = residual + gate[idx] * (x W^T + b): the block's closing gated residual
// (src/h3_flash/runtime/kernels/transformer.py:123-126) fused into the FFN output
// projection; idx = index[row % n_index] picks the AdaLN table row. The
// projection is not rounded to bf16 before the gated add.
struct GatedResidualEpi {
  static constexpr int kSegments = 2;
  static constexpr bool kStaged = false;
  static constexpr bool kTmaStore = false;
  __nv_bfloat16* out;
  int64_t ldo;
  const __nv_bfloat16* bias;      // [N] or nullptr
  const __nv_bfloat16* residual;  // [rows, N], row stride ldr
  int64_t ldr;
  const __nv_bfloat16* gate;      // [n_table, N], row stride ldg
  int64_t ldg;
  const int64_t* index;           // [n_index]
  int64_t n_index;

  template <class Put>
  __device__ __forceinline__ void fill(uint32_t tacc, int seg, int64_t row, int n0, Put put8) const {
    const __nv_bfloat16* res = residual + row * ldr;
    const __nv_bfloat16* g = gate + __ldg(index + row % n_index) * ldg;
#pragma unroll 1
    for (int q4 = 0; q4 < 4; ++q4) {
      float x[32];
      load32(tacc + (uint32_t)(seg * 128 + 32 * q4), x);
      const int col0 = n0 + seg * 128 + 32 * q4;
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const int col = col0 + 8 * c8;
        const f8 rv = unpack8(*reinterpret_cast<const uint4*>(res + col));
        const f8 gv = unpack8(ld_cached(g + col));
        f8 bv;
        if (bias != nullptr) bv = unpack8(ld_cached(bias + col));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float y = x[8 * c8 + j] + (bias != nullptr ? bv.v[j] : 0.f);
          x[8 * c8 + j] = rv.v[j] + gv.v[j] * y;
        }
        put8(4 * q4 + c8, x + 8 * c8);
      }
    }
  }
  __device__ __forceinline__ __nv_bfloat16* dest(int seg, int64_t row, int n0) const {
    return out + row * ldo + n0 + seg * 128;
  }
  __device__ __forceinline__ void finish() const {}
};

// SwiGLU on an interleaved projection: tile columns [0, 128) are value columns
// [128t, 128t+128) and tile columns [128, 256) the matching gate columns; the
// output is (value + b_v) * silu(gate + b_g) at output columns [128t, 128t+128).
struct SwigluEpi {
  static constexpr int kSegments = 1;
  static constexpr bool kStaged = false;
  static constexpr bool kTmaStore = false;
  __nv_bfloat16* out;
  int64_t ldo;
  const __nv_bfloat16* bias;  // interleaved like W, [2 n] or nullptr

  template <class Put>
  __device__ __forceinline__ void fill(uint32_t tacc, int, int64_t, int n0, Put put8) const {
#pragma unroll 1
    for (int q4 = 0; q4 < 4; ++q4) {
      float v[32], g[32];
      load32(tacc + (uint32_t)(32 * q4), v);
      load32(tacc + (uint32_t)(128 + 32 * q4), g);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        if (bias != nullptr) {
          const f8 bv = unpack8(ld_cached(bias + n0 + 32 * q4 + 8 * c8));
          const f8 bg = unpack8(ld_cached(bias + n0 + 128 + 32 * q4 + 8 * c8));
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            v[8 * c8 + j] += bv.v[j];
            g[8 * c8 + j] += bg.v[j];
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * c8 + j] *= silu(g[8 * c8 + j]);
        put8(4 * q4 + c8, v + 8 * c8);
      }
    }
  }
  __device__ __forceinline__ __nv_bfloat16* dest(int, int64_t row, int n0) const {
    return out + row * ldo + n0 / 2;
  }
  __device__ __forceinline__ void finish() const {}
};

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------

template <class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap x_map,
                const __grid_constant__ CUtensorMap w_map, const Shape prm,
                const __grid_constant__ Epi epi) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + kSmemBar;
  auto bar_full = [&](int s) { return bars + 8u * s; };
  auto bar_empty = [&](int s) { return bars + 8u * (kStages + s); };
  auto bar_tfull = [&](int b) { return bars + 8u * (2 * kStages + b); };
  auto bar_tempty = [&](int b) { return bars + 8u * (2 * kStages + 2 + b); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + kNumBars * 8);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const uint32_t cta = cluster_ctarank();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int n_tiles = prm.tiles_m * prm.tiles_n;
  const int k_blocks = prm.dim / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_tfull(b), 1);
      mbar_init(bar_tempty(b), 2 * kEpiWarps);  // every epilogue warp of both CTAs
    }
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {  // the same warp in both CTAs allocates, jointly
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    prefetch_map(&x_map);
    prefetch_map(&w_map);
  }
  tc_fence_before();
  cluster_sync_all();  // the peer's barriers exist before any remote arrival
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: this CTA's halves of x and W ----------------
      bool ok = true;
      int it = 0;
      for (int tile = pair; tile < n_tiles && ok; tile += n_pairs) {
        int tm, tn;
        tile_coords(tile, prm, tm, tn);
        const int m0 = tm * (2 * kBM) + (int)cta * kBM;
        const int n0 = tn * kBN + (int)cta * kBNc;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          ok = wait_bar(bar_empty(s), ((it / kStages) & 1) ^ 1, abort_flag, prm.status);
          if (!ok) break;
          if (cta == 0) mbar_expect_tx(bar_full(s), 2 * kStageBytes);
          const uint32_t full = map_to_cta(bar_full(s), 0);
          const uint32_t sa = sbase + s * kStageBytes;
          tma_load_2d_pair(sa, &x_map, full, kb * kBK, m0);
          tma_load_2d_pair(sa + kABytes, &w_map, full, kb * kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (cta == 0 && lane == 0) {
      // ---------------- MMA issuer for the pair ----------------
      bool ok = true;
      int it = 0, local = 0;
      const uint64_t desc0 = smem_desc(sbase, 16, 1024);
      for (int tile = pair; tile < n_tiles && ok; tile += n_pairs, ++local) {
        const int b = local & 1;
        ok = wait_bar(bar_tempty(b), ((local >> 1) & 1) ^ 1, abort_flag, prm.status);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(b * kBN);
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          ok = wait_bar(bar_full(s), (it / kStages) & 1, abort_flag, prm.status);
          if (!ok) break;
          tc_fence_after();
          const uint64_t a_desc = desc0 + (uint64_t)((s * kStageBytes) >> 4);
          const uint64_t b_desc = desc0 + (uint64_t)((s * kStageBytes + kABytes) >> 4);
          // K step kk of 16 elements: 32 bytes further inside the 128-byte swizzle row.
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_pair(d, a_desc + (uint64_t)((kk * 32) >> 4), b_desc + (uint64_t)((kk * 32) >> 4),
                     (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit_pair(bar_empty(s));  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        mma_commit_pair(bar_tfull(b));  // accumulator b complete
      }
    }
  } else {
    // ---------------- epilogue: one output row per thread, stores per warp ----------------
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
    uint8_t* stage = smem + kSmemEpi + (warp - 2) * kEpiStageBytes;
    // Staging layouts. Plain stores: chunk c (16 bytes) of staging row r sits at
    // position c ^ (r & 15) of the row's 256 bytes. TMA stores: two 64-column boxes of
    // 32 rows x 128 bytes in the 128-byte swizzle (chunk c % 8 of row r at position
    // (c % 8) ^ (r % 8)), one per half of the segment. Both keep the per-thread row
    // writes and the per-warp reads free of bank conflicts.
    uint8_t* my_row = stage + lane * kSegBytes;
    __nv_bfloat16* direct = nullptr;  // unstaged epilogues: this thread's row segment
    auto put8 = [&](int c, const float* v) {
      if constexpr (Epi::kTmaStore)
        *reinterpret_cast<uint4*>(stage + (c >> 3) * (kEpiStageBytes / 2) + lane * 128 +
                                  (((c & 7) ^ (lane & 7)) << 4)) = pack8(v);
      else if constexpr (Epi::kStaged)
        *reinterpret_cast<uint4*>(my_row + ((c ^ (lane & 15)) << 4)) = pack8(v);
      else if (direct != nullptr)
        *reinterpret_cast<uint4*>(direct + 8 * c) = pack8(v);
    };
    bool ok = true;
    int local = 0;
    for (int tile = pair; tile < n_tiles && ok; tile += n_pairs, ++local) {
      const int b = local & 1;
      ok = wait_bar(bar_tfull(b), (local >> 1) & 1, abort_flag, prm.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(tile, prm, tm, tn);
      const int64_t row0 = (int64_t)tm * (2 * kBM) + (int)cta * kBM + quad * 32;
      const int n0 = tn * kBN;
      const int64_t my = row0 + lane;
      const uint32_t tacc = tmem + lane_base + (uint32_t)(b * kBN);
#pragma unroll 1
      for (int seg = 0; seg < Epi::kSegments; ++seg) {
        // Rows past the end compute on the accumulator's padding rows (TMA filled
        // their x with zeros) and are never stored.
        if constexpr (!Epi::kStaged) direct = my < prm.rows ? epi.dest(seg, my, n0) : nullptr;
        if constexpr (Epi::kTmaStore) {
          // The previous segment's stores have read the staging buffer.
          if (lane == 0) bulk_wait_read();
          __syncwarp();
        }
        epi.fill(tacc, seg, my < prm.rows ? my : prm.rows - 1, n0, put8);
        if constexpr (Epi::kTmaStore) {
          // Rows past the end lie outside the tensor map: the TMA unit drops them.
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            const int col = n0 + seg * kHeadDim;
            tma_store_2d(&epi.out_map, smem_u32(stage), col, (int)row0);
            tma_store_2d(&epi.out_map, smem_u32(stage + kEpiStageBytes / 2), col + 64, (int)row0);
            bulk_commit();
          }
          continue;
        }
        if constexpr (!Epi::kStaged) continue;
        __syncwarp();
        // Two whole rows per instruction: lanes 0-15 row i, lanes 16-31 row i + 1.
#pragma unroll 4
        for (int i = 0; i < 32; i += 2) {
          const int r = i + (lane >> 4);
          const int c = lane & 15;
          const int64_t row = row0 + r;
          if (row < prm.rows) {
            const uint4 v = *reinterpret_cast<const uint4*>(stage + r * kSegBytes + ((c ^ (r & 15)) << 4));
            *reinterpret_cast<uint4*>(epi.dest(seg, row, n0) + 8 * c) = v;
          }
        }
        __syncwarp();
      }
      // Every segment is read out of accumulator b: hand it back to the MMA issuer.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_cta(bar_tempty(b), 0));
    }
    if constexpr (Epi::kTmaStore) {
      if (lane == 0) bulk_wait_all();
    }
    epi.finish();
  }

  if (*abort_flag) {
    // Let TMA copies and MMAs already issued land before shared memory and TMEM go.
    const unsigned long long t0 = globaltimer();
    while (globaltimer() - t0 < kDrainNs) __nanosleep(1000);
  }
  // Both CTAs are done with every TMEM and shared-memory access of the pair's
  // MMAs before either frees its TMEM or exits.
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// The RoPE tables in the QKV epilogue's layout: float4 slot s of row r at
// tab[s * rows + r], so that 32 consecutive rows of one slot are one 512-byte span.
// Rotary chunk k (16 rotate-half pairs, half = rot / 2) owns slots 16k .. 16k + 15:
// cos[16k, +16), sin[16k, +16), cos[half + 16k, +16), sin[half + 16k, +16).
__global__ void rope_tables_kernel(float4* __restrict__ tab, const float* __restrict__ cos,
                                   const float* __restrict__ sin, int64_t rows, int rot) {
  const int half = rot / 2;
  const int64_t n = rows * half;  // rot / 2 slots per row
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int s = (int)(i / rows);
    const int64_t r = i - (int64_t)s * rows;
    const int k = s >> 4, j = s & 15;
    const float* src = (j & 4) ? sin : cos;
    const int col = ((j & 8) ? half : 0) + 16 * k + 4 * (j & 3);
    tab[i] = __ldg(reinterpret_cast<const float4*>(src + r * rot + col));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D map over (K, rows) of a row-major bf16 matrix with a (64, 128) box.
int make_map(CUtensorMap* map, const void* base, int64_t k, int64_t rows, int64_t row_stride,
             const char* name) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("h3b_gemm: cuTensorMapEncodeTiled is unavailable");
    return H3B_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "h3b_gemm: tensor map for %s rejected (CUresult %d)",
             name, (int)r);
    set_error(buf);
    return H3B_ERR_CUDA;
  }
  return H3B_OK;
}

// 2-D map over (N, rows) of the bf16 output, row stride ldo, with the epilogue's
// (64, 32) store box in the 128-byte swizzle.
int make_out_map(CUtensorMap* map, void* out, int64_t n, int64_t rows, int64_t ldo) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("h3b_gemm: cuTensorMapEncodeTiled is unavailable");
    return H3B_ERR_CUDA;
  }
  cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ldo * 2};
  cuuint32_t box[2] = {64, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, out, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "h3b_gemm: tensor map for out rejected (CUresult %d)", (int)r);
    set_error(buf);
    return H3B_ERR_CUDA;
  }
  return H3B_OK;
}

// Tensor maps, shape and grid of one call.
struct Common {
  CUtensorMap xm, wm;
  Shape shape;
  int grid;
};

// Checks shared by every entry point and the tensor maps of x [rows, dim] and
// W [n, dim] (both K-major). `what` names the entry point in errors.
int prepare(Common& c, const char* what, const void* x, int64_t rows, int64_t dim,
            int64_t x_row_stride, const void* w, int64_t n) {
  char msg[256];
  if (rows < 0 || dim <= 0 || n <= 0) {
    snprintf(msg, sizeof(msg), "%s: bad shape", what);
    set_error(msg);
    return H3B_ERR_VALUE;
  }
  if (dim % kBK != 0 || n % kBN != 0) {
    snprintf(msg, sizeof(msg), "%s: needs dim %% 64 == 0 and output columns %% 256 == 0", what);
    set_error(msg);
    return H3B_ERR_UNSUPPORTED;
  }
  if (rows >= (1LL << 31) || dim >= (1LL << 31) || n >= (1LL << 31)) {
    snprintf(msg, sizeof(msg), "%s: shape exceeds limits", what);
    set_error(msg);
    return H3B_ERR_VALUE;
  }
  if (rows == 0) return H3B_OK;  // nothing to project; empty tensors may carry null pointers
  if (x == nullptr || w == nullptr || !aligned16(x) || !aligned16(w) || x_row_stride < dim ||
      x_row_stride % 8 != 0) {
    snprintf(msg, sizeof(msg),
             "%s: x and W must be 16-byte aligned, x row stride >= dim and a multiple of 8", what);
    set_error(msg);
    return H3B_ERR_VALUE;
  }
  int rc;
  if ((rc = make_map(&c.xm, x, dim, rows, x_row_stride, "x")) != H3B_OK) return rc;
  if ((rc = make_map(&c.wm, w, dim, n, dim, "w")) != H3B_OK) return rc;
  c.shape.rows = rows;
  c.shape.dim = (int)dim;
  c.shape.tiles_m = (int)((rows + 2 * kBM - 1) / (2 * kBM));
  c.shape.tiles_n = (int)(n / kBN);
  // Raster groups: a W panel of group_n tile columns is group_n * 256 * dim * 2
  // bytes. Grouping reads x once per group instead of once, so it pays when W is
  // wide and its tile columns are cheap (short K): then a ~32 MB panel (a quarter
  // of L2) survives the x and output traffic around it. Otherwise (all of W fits
  // in a third of L2, or a long K makes x the larger stream) tiles stay row-major.
  {
    const int64_t panel = (int64_t)kBN * dim * 2;
    const int64_t budget = 32ll << 20;
    int g = c.shape.tiles_n;
    if ((int64_t)c.shape.tiles_n * panel > 48ll << 20 && panel <= (2ll << 20))
      g = (int)(budget / panel);
    c.shape.group_n = g < 1 ? 1 : (g > c.shape.tiles_n ? c.shape.tiles_n : g);
  }
  c.shape.status = status_ptr();
  if (c.shape.status == nullptr) {
    snprintf(msg, sizeof(msg), "%s: cannot resolve the device status word", what);
    set_error(msg);
    return H3B_ERR_CUDA;
  }
  const int tiles = c.shape.tiles_m * c.shape.tiles_n;
  const int pairs = num_sms() / 2;
  c.grid = 2 * (tiles < pairs ? tiles : pairs);
  return H3B_OK;
}

template <class Epi>
int launch(const Common& c, const Epi& epi, const char* what, cudaStream_t stream) {
  // Set once per device and context (a function attribute belongs to the context).
  static ContextSlot attr_slots[kMaxDevices];
  cudaError_t e = cudaErrorInvalidDevice;
  if (context_cached(attr_slots, [&]() -> void* {
        e = cudaFuncSetAttribute(gemm_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmemAlloc);
        return e == cudaSuccess ? reinterpret_cast<void*>(1) : nullptr;
      }) == nullptr) {
    set_error(std::string(what) + ": cannot reserve shared memory: " + cudaGetErrorString(e));
    return H3B_ERR_CUDA;
  }
  gemm_kernel<Epi><<<(unsigned)c.grid, kThreads, kSmemAlloc, stream>>>(c.xm, c.wm, c.shape, epi);
  return check_launch(what);
}

// QKV epilogue arguments (both QKV entry points): the RoPE tables are relaid into
// the workspace first, on the same stream.
template <class Dst>
int launch_qkv(const Common& c, const Dst& d, const void* bias, const void* q_weight,
               const void* k_weight, const float* cos, const float* sin, int64_t rows,
               int64_t heads, int64_t rot, float q_eps, float k_eps, void* workspace,
               cudaStream_t stream) {
  auto* tab = static_cast<float4*>(workspace);
  if (rot > 0) {
    const int64_t n = rows * (rot / 2);
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
    rope_tables_kernel<<<blocks, 256, 0, stream>>>(tab, cos, sin, rows, (int)rot);
    const int rc = check_launch("h3b_qkv_gemm_pack");
    if (rc != H3B_OK) return rc;
  }
  auto go = [&](auto rot_tag) {
    constexpr int R = decltype(rot_tag)::value;
    QkvEpi<R, Dst> epi{static_cast<const __nv_bfloat16*>(bias),
                       static_cast<const __nv_bfloat16*>(q_weight),
                       static_cast<const __nv_bfloat16*>(k_weight), tab, rows, q_eps, k_eps,
                       (int)heads, d};
    return launch(c, epi, "h3b_qkv_gemm_pack", stream);
  };
  switch (rot) {
    case 0: return go(std::integral_constant<int, 0>{});
    case 64: return go(std::integral_constant<int, 64>{});
    case 96: return go(std::integral_constant<int, 96>{});
    default: return go(std::integral_constant<int, 128>{});
  }
}

int64_t qkv_workspace_bytes(int64_t rows, int64_t rotary_dim) {
  return rows * rotary_dim * 2 * (int64_t)sizeof(float);
}

// Shape checks of the QKV entry points (before the no-rows early return) ...
int check_qkv_shape(int64_t heads, int64_t head_dim, int64_t rotary_dim) {
  if (head_dim != kHeadDim || heads <= 0 || (heads * kHeadDim) % kBN != 0) {
    set_error("h3b_qkv_gemm_pack: needs head_dim 128, an even head count and dim % 64 == 0");
    return H3B_ERR_UNSUPPORTED;
  }
  if (!(rotary_dim == 0 || rotary_dim == 64 || rotary_dim == 96 || rotary_dim == 128)) {
    set_error("h3b_qkv_gemm_pack: rotary dimension must be 0, 64, 96 or 128");
    return H3B_ERR_UNSUPPORTED;
  }
  return H3B_OK;
}

// ... and their pointer checks (after it: empty tensors may carry null pointers).
int check_qkv(const void* bias, const void* q_weight, const void* k_weight, const float* cos,
              const float* sin, int64_t rows, int64_t rotary_dim, const void* workspace,
              int64_t workspace_bytes) {
  H3B_REQUIRE(q_weight != nullptr && k_weight != nullptr, "qkv_gemm_pack: null argument");
  H3B_REQUIRE(rotary_dim == 0 || (cos != nullptr && sin != nullptr),
              "qkv_gemm_pack: rotary tables missing");
  H3B_REQUIRE((bias == nullptr || aligned16(bias)) && aligned16(q_weight) && aligned16(k_weight) &&
                  (rotary_dim == 0 || (aligned16(cos) && aligned16(sin))),
              "qkv_gemm_pack: buffers must be 16-byte aligned");
  const int64_t need = qkv_workspace_bytes(rows, rotary_dim);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) {
    char buf[200];
    snprintf(buf, sizeof(buf),
             "h3b_qkv_gemm_pack: needs a 16-byte aligned workspace of %lld bytes for the RoPE "
             "tables (got %lld)",
             (long long)need, (long long)(workspace == nullptr ? 0 : workspace_bytes));
    set_error(buf);
    return H3B_ERR_VALUE;
  }
  return H3B_OK;
}

}  // namespace gemm
}  // namespace h3b

using namespace h3b;
using namespace h3b::gemm;

extern "C" int h3b_qkv_gemm_pack(void* send, int64_t world, const void* x, int64_t rows,
                                 int64_t dim, int64_t x_row_stride, const void* w_qkv,
                                 const void* bias, const void* q_weight, const void* k_weight,
                                 const float* cos, const float* sin, int64_t heads,
                                 int64_t head_dim, int64_t rotary_dim, float q_eps, float k_eps,
                                 void* workspace, int64_t workspace_bytes, h3b_stream_t stream) {
  H3B_REQUIRE(world >= 1 && heads > 0 && heads % world == 0,
              "heads (%lld) must divide Ulysses degree (%lld)", (long long)heads, (long long)world);
  H3B_REQUIRE(rows >= 0 && dim > 0, "qkv_gemm_pack: bad shape");
  int rc = check_qkv_shape(heads, head_dim, rotary_dim);
  if (rc != H3B_OK || rows == 0) return rc;
  rc = check_qkv(bias, q_weight, k_weight, cos, sin, rows, rotary_dim, workspace, workspace_bytes);
  if (rc != H3B_OK) return rc;
  Common c;
  rc = prepare(c, "h3b_qkv_gemm_pack", x, rows, dim, x_row_stride, w_qkv, 3 * heads * kHeadDim);
  if (rc != H3B_OK) return rc;
  H3B_REQUIRE(send != nullptr && aligned16(send), "qkv_gemm_pack: send must be 16-byte aligned");
  LocalSend d{static_cast<__nv_bfloat16*>(send), rows, (int)(heads / world)};
  return launch_qkv(c, d, bias, q_weight, k_weight, cos, sin, rows, heads, rotary_dim, q_eps,
                    k_eps, workspace, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_qkv_gemm_pack_p2p(void* const* recv_ptrs, int64_t world, int64_t row_offset,
                                     int64_t total_rows, const void* x, int64_t rows,
                                     int64_t dim, int64_t x_row_stride, const void* w_qkv,
                                     const void* bias, const void* q_weight,
                                     const void* k_weight, const float* cos, const float* sin,
                                     int64_t heads, int64_t head_dim, int64_t rotary_dim,
                                     float q_eps, float k_eps, void* workspace,
                                     int64_t workspace_bytes, h3b_stream_t stream) {
  H3B_REQUIRE(world >= 1 && world <= kMaxPeers && heads > 0 && heads % world == 0,
              "heads (%lld) must divide Ulysses degree (%lld), world <= %d", (long long)heads,
              (long long)world, kMaxPeers);
  H3B_REQUIRE(recv_ptrs != nullptr, "qkv_gemm_pack_p2p: null pointer array");
  H3B_REQUIRE(row_offset >= 0 && rows >= 0 && row_offset + rows <= total_rows,
              "qkv_gemm_pack_p2p: rows [%lld, %lld) outside the %lld-row request",
              (long long)row_offset, (long long)(row_offset + rows), (long long)total_rows);
  H3B_REQUIRE(dim > 0, "qkv_gemm_pack: bad shape");
  int rc = check_qkv_shape(heads, head_dim, rotary_dim);
  if (rc != H3B_OK || rows == 0) return rc;
  rc = check_qkv(bias, q_weight, k_weight, cos, sin, rows, rotary_dim, workspace, workspace_bytes);
  if (rc != H3B_OK) return rc;
  Common c;
  rc = prepare(c, "h3b_qkv_gemm_pack_p2p", x, rows, dim, x_row_stride, w_qkv,
               3 * heads * kHeadDim);
  if (rc != H3B_OK) return rc;
  PeerRecv d;
  memset(&d, 0, sizeof(d));
  for (int i = 0; i < world; ++i) {
    H3B_REQUIRE(recv_ptrs[i] != nullptr && aligned16(recv_ptrs[i]),
                "qkv_gemm_pack_p2p: receive buffer of rank %d is null or not 16-byte aligned", i);
    d.recv.p[i] = recv_ptrs[i];
  }
  d.row_offset = row_offset;
  d.hl = (int)(heads / world);
  return launch_qkv(c, d, bias, q_weight, k_weight, cos, sin, rows, heads, rotary_dim, q_eps,
                    k_eps, workspace, static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_qkv_gemm_pack_workspace_size(int64_t rows, int64_t rotary_dim,
                                                int64_t* bytes_out) {
  H3B_REQUIRE(bytes_out != nullptr, "qkv_gemm_pack_workspace_size: null output pointer");
  H3B_REQUIRE(rows >= 0 && rotary_dim >= 0, "qkv_gemm_pack_workspace_size: negative shape");
  *bytes_out = qkv_workspace_bytes(rows, rotary_dim);
  return H3B_OK;
}

extern "C" int h3b_gemm(void* out, int64_t out_row_stride, const void* x, int64_t rows,
                        int64_t dim, int64_t x_row_stride, const void* w, int64_t n,
                        const void* bias, int64_t activation, h3b_stream_t stream) {
  H3B_REQUIRE(activation == kActNone || activation == kActGeluTanh,
              "gemm: activation must be 0 (none) or 1 (gelu-tanh)");
  Common c;
  int rc = prepare(c, "h3b_gemm", x, rows, dim, x_row_stride, w, n);
  if (rc != H3B_OK || rows == 0) return rc;
  H3B_REQUIRE(out != nullptr && aligned16(out) && out_row_stride >= n && out_row_stride % 8 == 0,
              "gemm: out must be 16-byte aligned with a row stride >= n and a multiple of 8");
  H3B_REQUIRE(bias == nullptr || aligned16(bias), "gemm: bias must be 16-byte aligned");
  auto* o = static_cast<__nv_bfloat16*>(out);
  auto* b = static_cast<const __nv_bfloat16*>(bias);
  const auto s = static_cast<cudaStream_t>(stream);
  CUtensorMap om;
  if ((rc = make_out_map(&om, out, n, rows, out_row_stride)) != H3B_OK) return rc;
  if (activation == kActGeluTanh)
    return launch(c, DenseEpi<kActGeluTanh>{om, o, out_row_stride, b}, "h3b_gemm", s);
  return launch(c, DenseEpi<kActNone>{om, o, out_row_stride, b}, "h3b_gemm", s);
}

extern "C" int h3b_gemm_swiglu(void* out, int64_t out_row_stride, const void* x, int64_t rows,
                               int64_t dim, int64_t x_row_stride, const void* w_interleaved,
                               int64_t n_out, const void* bias_interleaved,
                               h3b_stream_t stream) {
  H3B_REQUIRE(n_out > 0 && n_out % 128 == 0, "gemm_swiglu: output width must be a multiple of 128");
  Common c;
  int rc = prepare(c, "h3b_gemm_swiglu", x, rows, dim, x_row_stride, w_interleaved, 2 * n_out);
  if (rc != H3B_OK || rows == 0) return rc;
  H3B_REQUIRE(out != nullptr && aligned16(out) && out_row_stride >= n_out && out_row_stride % 8 == 0,
              "gemm_swiglu: out must be 16-byte aligned with a row stride >= n and a multiple of 8");
  H3B_REQUIRE(bias_interleaved == nullptr || aligned16(bias_interleaved),
              "gemm_swiglu: bias must be 16-byte aligned");
  SwigluEpi epi{static_cast<__nv_bfloat16*>(out), out_row_stride,
                static_cast<const __nv_bfloat16*>(bias_interleaved)};
  return launch(c, epi, "h3b_gemm_swiglu", static_cast<cudaStream_t>(stream));
}

extern "C" int h3b_gemm_gated_residual(void* out, int64_t out_row_stride, const void* x,
                                       int64_t rows, int64_t dim, int64_t x_row_stride,
                                       const void* w, int64_t n, const void* bias,
                                       const void* residual, int64_t residual_row_stride,
                                       const void* gate, int64_t gate_row_stride,
                                       const int64_t* index, int64_t n_index,
                                       h3b_stream_t stream) {
  Common c;
  int rc = prepare(c, "h3b_gemm_gated_residual", x, rows, dim, x_row_stride, w, n);
  if (rc != H3B_OK || rows == 0) return rc;
  H3B_REQUIRE(out != nullptr && aligned16(out) && out_row_stride >= n && out_row_stride % 8 == 0,
              "gemm_gated_residual: out must be 16-byte aligned with a row stride >= n and a "
              "multiple of 8");
  H3B_REQUIRE(residual != nullptr && aligned16(residual) && residual_row_stride >= n &&
                  residual_row_stride % 8 == 0,
              "gemm_gated_residual: residual must be 16-byte aligned with a row stride >= n and a "
              "multiple of 8");
  H3B_REQUIRE(gate != nullptr && aligned16(gate) && gate_row_stride % 8 == 0,
              "gemm_gated_residual: gate table must be 16-byte aligned, row stride a multiple of 8");
  H3B_REQUIRE(index != nullptr && n_index > 0, "gemm_gated_residual: empty index");
  H3B_REQUIRE(bias == nullptr || aligned16(bias), "gemm_gated_residual: bias must be 16-byte aligned");
  GatedResidualEpi epi{static_cast<__nv_bfloat16*>(out), out_row_stride,
                       static_cast<const __nv_bfloat16*>(bias),
                       static_cast<const __nv_bfloat16*>(residual), residual_row_stride,
                       static_cast<const __nv_bfloat16*>(gate), gate_row_stride, index, n_index};
  return launch(c, epi, "h3b_gemm_gated_residual", static_cast<cudaStream_t>(stream));
}
