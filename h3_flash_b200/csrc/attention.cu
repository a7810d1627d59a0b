// Dense non-causal attention for B200 (sm_100a): tcgen05 MMA with TMEM
// accumulators, TMA-fed shared-memory operands, fp32 online softmax.
//
// One CTA owns two 128-row query tiles of one (batch, head) and streams the
// whole key/value sequence in 128-row blocks:
//
//   warp 8      TMA producer: Q0, Q1 once, then K_j and V_j together into a
//               two-stage ring (64 KB per stage, 128B-swizzled), one mbarrier
//               per stage for both: the MMA warp waits once per key block.
//   warp 9      MMA issuer: the whole warp runs the issue loop (waits, descriptor
//               arithmetic) and one elected lane issues: S_t = Q_t K_j^T into
//               TMEM, then O_t += P_t V_j with P_t read from TMEM (A operand) and
//               V_j from shared memory (MN-major B operand), in two 64-key halves.
//               Tiles t=0,1 alternate, so the tensor core works on one tile
//               while the other tile's softmax runs.
//   warps 0-3   softmax of tile 0, warps 4-7 softmax of tile 1. Warp w owns
//               TMEM lane quadrant w%4, and each of its threads owns one query
//               row: it loads the row's 128 scores of a block from TMEM, takes
//               the row max itself (no exchange between threads), computes
//               p = 2^(s*c - m), writes P (bf16) over the S columns it has
//               read and keeps the row sum in fp32. Exponentials use MUFU
//               ex2 (a polynomial on the FMA pipe for part of them is a build
//               option, off by default: slower here). O is rescaled in TMEM
//               only when the running max grows by more than 2^8 (P stays
//               <= 256, exact in the fp32 accumulator), which after the first
//               blocks is rare.
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// P of tile t, keys [64h, 64h+64), lives in S_t columns [32h, 32h+32): key k
// in column k/2 (even key in the low half), the layout the TS-form MMA reads.
// A tcgen05.commit tracks every earlier MMA of the issuing thread, so the
// commit after S_t(j) also certifies that PV_t(j-1) is done: the softmax may
// touch O_t once it has seen S_t(j).
//
// Output: the local [B, S, H, D] tensor, or (h3b_attention_p2p) the merged
// buffers of the ranks that own the rows. There the epilogue stores each
// finished row of local head h over NVLink into its owner's [rows, H, D] buffer
// at head rank*hl + h: the output all-to-all and the head merge of packed
// Ulysses run inside the attention kernel, tile by tile, while later tiles
// are still computing.
//
// Every mbarrier wait is bounded by a wall-clock limit. On expiry the thread
// ORs kStatusAttentionTimeout into the library status word, raises the CTA
// abort flag and unwinds; the other roles see the flag in their own waits, so
// the CTA frees its TMEM and exits instead of hanging the GPU.
//
// Replaces torch SDPA in src/h3_flash/runtime/parallel/packed_ulysses.py:201-209
// and the FA4 call in src/h3_flash/runtime/attention/dense_fa4.py:74-81.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace h3b {
namespace attn {

constexpr int kBlockM = 128;  // query rows per tile
constexpr int kBlockN = 128;  // key rows per block
constexpr int kHeadDim = 128;
constexpr int kTiles = 2;  // query tiles per CTA
constexpr int kStages = 2;  // K/V ring depth (one stage holds K_j and V_j)
constexpr int kSoftmaxWarps = 4 * kTiles;  // one per TMEM lane quadrant per tile
constexpr int kThreads = (kSoftmaxWarps + 2) * 32;  // + TMA warp + MMA warp
constexpr int kLoadWarp = kSoftmaxWarps;
constexpr int kMmaWarp = kSoftmaxWarps + 1;

constexpr uint32_t kTileBytes = kBlockM * kHeadDim * 2;  // 32 KB: two 16 KB swizzled halves
constexpr uint32_t kHalfBytes = kTileBytes / 2;
constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemK = kSmemQ + kTiles * kTileBytes;
constexpr uint32_t kSmemV = kSmemK + kStages * kTileBytes;
constexpr uint32_t kSmemBar = kSmemV + kStages * kTileBytes;
// barriers: q[2], kvfull[stages], kvempty[stages], s[2], p[2][2], o[2] + tmem slot + abort
constexpr uint32_t kNumBars = kTiles + 2 * kStages + 4 * kTiles;
constexpr uint32_t kSmemBytes = kSmemBar + ((kNumBars * 8 + 16 + 127) / 128) * 128;
constexpr uint32_t kSmemAlloc = kSmemBytes + 1024;  // slack to 1024-align the base
static_assert(kSmemAlloc <= 232448, "shared memory per CTA");

constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0;    // + t*128
constexpr uint32_t kTmemO = 256;  // + t*128

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// Rescale O only when the running row max (log2 units) grew by more than this.
constexpr float kRescaleThreshold = 8.0f;

// Of every 8 column pairs of a row, this many take the FMA-pipe exp2
// (exp2_poly) instead of MUFU ex2. The MUFU time of one tile's softmax is
// close to the tensor time of the other tile's MMAs, which the offload
// shortens; but in this kernel the softmax finishes ahead of the MMA warp and
// the extra FMA-pipe instructions slow the SMSP that issues the MMAs, so the
// measured optimum is 0 (kept as a build-time knob).
#ifndef H3B_ATTN_POLY_PAIRS
#define H3B_ATTN_POLY_PAIRS 0
#endif
constexpr int kPolyPairs = H3B_ATTN_POLY_PAIRS;

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

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity. Returns false if the CTA
// aborted (another thread timed out) or this wait itself timed out.
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
        if (status) atomicOr(status, kStatusAttentionTimeout);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
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
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M=128, N=128.
// b_mn_major selects an MN-major B operand (V in P.V).
__host__ __device__ constexpr uint32_t instr_desc(bool b_mn_major) {
  return (1u << 4)                   // D format f32
         | (1u << 7)                 // A bf16
         | (1u << 10)                // B bf16
         | ((b_mn_major ? 1u : 0u) << 16)
         | ((uint32_t)(kBlockN >> 3) << 17)  // N >> 3
         | ((uint32_t)(kBlockM >> 4) << 24); // M >> 4
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// One lane of a converged warp (elect.sync over all 32 lanes elects the lowest,
// lane 0, every time): the lane that issues the warp's MMAs and commits. A
// commit only tracks MMAs of its own thread, so both must come from that lane.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
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

// Waits for this thread's outstanding tcgen05.ld and pins the 32 registers
// after the wait so no use is scheduled above it.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
  asm volatile(""
               : "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]),
                 "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
                 "+r"(r[31]));
}
__device__ __forceinline__ void tmem_pin(uint32_t (&r)[32]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
  asm volatile(""
               : "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]),
                 "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
                 "+r"(r[31]));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// 32 lanes x 16 columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait16(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}

__device__ __forceinline__ void tmem_pin16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]);

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

// bar.sync on a named barrier shared by `count` threads (a multiple of 32).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Keys at block columns >= valid do not exist (sequence tail): score -inf.
__device__ __forceinline__ void mask_keys(uint32_t (&r)[32], int col0, int valid) {
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (col0 + i >= valid) r[i] = __float_as_uint(-INFINITY);
}

__device__ __forceinline__ void mask_keys16(uint32_t (&r)[16], int col0, int valid) {
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (col0 + i >= valid) r[i] = __float_as_uint(-INFINITY);
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair of fp32 values on the FMA pipe (no MUFU):
//   n = round(x) via the 1.5*2^23 shifter, f = x - n in [-1/2, 1/2],
//   2^f ~ c0 + f(c1 + f(c2 + f c3)), then n is added to the exponent field.
// The cubic is this file's own relative-error minimax fit of 2^f on [-1/2, 1/2]
// (Lawson-weighted least squares over Chebyshev points): max relative error
// 7.5e-5, below half a bf16 ulp (2^-9) of the P operand it feeds. Inputs are
// clamped to >= -126 so the exponent add never wraps (masked -inf keys become
// ~1e-38 instead of 0; their V rows are zero).
__device__ __forceinline__ float2 exp2_poly(float2 x) {
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float kShift = 12582912.f;  // 1.5 * 2^23
  const float2 t = __fadd2_rn(x, make_float2(kShift, kShift));
  const float2 n = __fadd2_rn(t, make_float2(-kShift, -kShift));
  const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(f, make_float2(0.0551716685f, 0.0551716685f),
                        make_float2(0.2426111400f, 0.2426111400f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677f, 0.6932609677f));
  p = __ffma2_rn(p, f, make_float2(0.9999280572f, 0.9999280572f));
  float2 r;
  r.x = __int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23));
  r.y = __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23));
  return r;
}

// ---------------------------------------------------------------------------
// Kernel
// ---------------------------------------------------------------------------

// Where output rows go when they leave this rank: the merged buffer
// dst[o] = [rows_o, heads_total, D] of the rank o that owns global row s
// (start[o] <= s < start[o+1]), at head head_base + h. world == 0: local out.
struct OutRoute {
  PeerPtrs dst;
  int64_t start[kMaxPeers + 1];
  int world, head_base, heads_total;
};

struct Params {
  __nv_bfloat16* out;
  int64_t o_batch_stride, o_row_stride, o_head_stride;
  OutRoute route;
  int seq_q, seq_k;
  float scale_log2;  // softmax_scale * log2(e)
  unsigned int* status;
  // Work decomposition. A unit is (batch, head, 256-row query block). Units
  // [0, n_full) run whole; each later unit runs as `splits` CTAs over
  // consecutive key ranges of `blocks_per_split` blocks, writing unnormalised
  // fp32 O and (max, sum) per row to `ws` for attention_combine.
  int heads, units_per_bh, n_full, splits, blocks_per_split;
  float* ws;
};

// First element of output row `row`, head `head`.
__device__ __forceinline__ __nv_bfloat16* out_row(const Params& prm, int batch, int row,
                                                  int head) {
  if (prm.route.world == 0)
    return prm.out + (int64_t)batch * prm.o_batch_stride + (int64_t)row * prm.o_row_stride +
           (int64_t)head * prm.o_head_stride;
  // Owner = last rank whose first row is <= row (starts never decrease).
  int owner = 0;
  int64_t first = 0;
#pragma unroll
  for (int j = 1; j < kMaxPeers; ++j)
    if (j < prm.route.world && row >= prm.route.start[j]) owner = j, first = prm.route.start[j];
  return reinterpret_cast<__nv_bfloat16*>(peer_at(prm.route.dst, owner)) +
         ((row - first) * prm.route.heads_total + prm.route.head_base + head) * kHeadDim;
}

// Workspace floats per split CTA: per tile, O [128 x 128] then (m, l) [128 x 2].
constexpr int kWsTileFloats = kBlockM * kHeadDim + 2 * kBlockM;
constexpr int kWsSlotFloats = kTiles * kWsTileFloats;

__global__ void __launch_bounds__(kThreads, 1)
    attention_fwd(const __grid_constant__ CUtensorMap q_map,
                  const __grid_constant__ CUtensorMap k_map,
                  const __grid_constant__ CUtensorMap v_map, const Params prm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase + kSmemQ;
  const uint32_t sK = sbase + kSmemK;
  const uint32_t sV = sbase + kSmemV;
  const uint32_t bars = sbase + kSmemBar;
  auto bar_q = [&](int t) { return bars + 8u * t; };
  // bar_kvfull(s): K_j and V_j of stage s landed; bar_kvempty(s): every MMA that
  // reads stage s (S of both tiles for K, PV of both tiles for V) is done.
  auto bar_kvfull = [&](int s) { return bars + 8u * (kTiles + s); };
  auto bar_kvempty = [&](int s) { return bars + 8u * (kTiles + kStages + s); };
  auto bar_s = [&](int t) { return bars + 8u * (kTiles + 2 * kStages + t); };
  // bar_p(t, h): the softmax of tile t has written P for keys [64h, 64h+64) of the block.
  auto bar_p = [&](int t, int h) { return bars + 8u * (kTiles + 2 * kStages + kTiles + 2 * t + h); };
  auto bar_o = [&](int t) { return bars + 8u * (kTiles + 2 * kStages + 3 * kTiles + t); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + kNumBars * 8);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_kv_total = (prm.seq_k + kBlockN - 1) / kBlockN;
  int unit = blockIdx.x, j0 = 0, n_kv = n_kv_total, split_slot = -1;
  if ((int)blockIdx.x >= prm.n_full) {
    const int r = blockIdx.x - prm.n_full;
    unit = prm.n_full + r / prm.splits;
    j0 = (r % prm.splits) * prm.blocks_per_split;
    n_kv = min(n_kv_total - j0, prm.blocks_per_split);
    split_slot = r;
  }
  const int qb = unit % prm.units_per_bh;
  const int bh = unit / prm.units_per_bh;
  const int head = bh % prm.heads;
  const int batch = bh / prm.heads;
  const int q_row0 = qb * (kTiles * kBlockM);

  if (threadIdx.x == 0) {
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(bar_q(t), 1);
      mbar_init(bar_s(t), 1);
      mbar_init(bar_p(t, 0), 4 * 32);
      mbar_init(bar_p(t, 1), 4 * 32);
      mbar_init(bar_o(t), 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_kvfull(s), 1);
      mbar_init(bar_kvempty(s), 1);
    }
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp == kLoadWarp && lane == 0) {
    prefetch_map(&q_map);
    prefetch_map(&k_map);
    prefetch_map(&v_map);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kLoadWarp) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      bool ok = true;
      for (int t = 0; t < kTiles; ++t) {
        mbar_expect_tx(bar_q(t), kTileBytes);
        const uint32_t dst = sQ + t * kTileBytes;
        const int row = q_row0 + t * kBlockM;
        tma_load_4d(dst, &q_map, bar_q(t), 0, head, row, batch);
        tma_load_4d(dst + kHalfBytes, &q_map, bar_q(t), 64, head, row, batch);
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % kStages;
        ok = wait_bar(bar_kvempty(st), ((j / kStages) & 1) ^ 1, abort_flag, prm.status);
        if (!ok) break;
        mbar_expect_tx(bar_kvfull(st), 2 * kTileBytes);
        const uint32_t kdst = sK + st * kTileBytes;
        const uint32_t vdst = sV + st * kTileBytes;
        const int key0 = (j0 + j) * kBlockN;
        tma_load_4d(kdst, &k_map, bar_kvfull(st), 0, head, key0, batch);
        tma_load_4d(kdst + kHalfBytes, &k_map, bar_kvfull(st), 64, head, key0, batch);
        tma_load_4d(vdst, &v_map, bar_kvfull(st), 0, head, key0, batch);
        tma_load_4d(vdst + kHalfBytes, &v_map, bar_kvfull(st), 64, head, key0, batch);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    // The whole warp runs the loop (every wait, all descriptor arithmetic, so the
    // operands are warp-uniform) and one elected lane issues each group of MMAs.
    // A single issuing thread must keep a shallow tensor-core queue fed, so the
    // loop waits on as few barriers per key block as it can: one for K_j and V_j
    // together, two for the P halves of each tile.
    constexpr uint32_t idesc_qk = instr_desc(false);
    constexpr uint32_t idesc_pv = instr_desc(true);
    auto wait_all = [&](uint32_t bar, uint32_t parity) -> bool {
      return __all_sync(0xffffffffu, wait_bar(bar, parity, abort_flag, prm.status));
    };
    bool ok = true;
    for (int t = 0; t < kTiles && ok; ++t) ok = wait_all(bar_q(t), 0);
    // Descriptors are built once: the loop only adds compile-time K-step offsets.
    // K-major SW128 tiles: K step kk sits at (kk/4) * 16 KB + (kk%4) * 32 B.
    // MN-major V tile: K step kk (16 keys) sits at kk * 2 KB; N halves 16 KB apart.
    // (The address field is the low 14 bits of (addr >> 4); every operand lies
    // below 256 KB, so adding an address delta >> 4 never carries out of it.)
    const uint64_t q_desc0 = smem_desc(sQ, 16, 1024);
    const uint64_t k_desc0 = smem_desc(sK, 16, 1024);
    const uint64_t v_desc0 = smem_desc(sV, kHalfBytes, 1024);
    // S_t = Q_t K_j^T : 8 MMAs of K=16 over the 128 head dims, then its commit.
    auto issue_s = [&](int t, int j) {
      const uint64_t qd = q_desc0 + (uint64_t)((t * kTileBytes) >> 4);
      const uint64_t kd = k_desc0 + (uint64_t)(((j % kStages) * kTileBytes) >> 4);
      const uint32_t d = tmem + kTmemS + t * 128;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
          const uint64_t off = (uint64_t)(((kk >> 2) * kHalfBytes + (kk & 3) * 32) >> 4);
          mma_ss(d, qd + off, kd + off, idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar_s(t));
      }
      __syncwarp();
    };
    // O_t += P_t V_j over keys [64h, 64h+64): 4 MMAs of K=16; P of keys
    // [16kk, 16kk+16) is S_t columns [8kk, 8kk+8).
    auto issue_pv = [&](int t, int j, int h) {
      const uint64_t vd = v_desc0 + (uint64_t)(((j % kStages) * kTileBytes) >> 4);
      const uint32_t d = tmem + kTmemO + t * 128;
      if (elect_one()) {
#pragma unroll
        for (int k4 = 0; k4 < kBlockN / 32; ++k4) {
          const int kk = h * (kBlockN / 32) + k4;
          mma_ts(d, tmem + kTmemS + t * 128 + kk * 8, vd + (uint64_t)((kk * 2048) >> 4), idesc_pv,
                 (j > 0 || kk > 0) ? 1u : 0u);
        }
      }
      __syncwarp();
    };
    auto commit = [&](uint32_t bar) {
      if (elect_one()) mma_commit(bar);
      __syncwarp();
    };
    if (ok) ok = wait_all(bar_kvfull(0), 0);
    if (ok) {
      tc_fence_after();
      for (int t = 0; t < kTiles; ++t) issue_s(t, 0);
    }
    for (int j = 0; j < n_kv && ok; ++j) {
      for (int t = 0; t < kTiles && ok; ++t) {
        ok = wait_all(bar_p(t, 0), j & 1);
        if (!ok) break;
        tc_fence_after();
        issue_pv(t, j, 0);
        ok = wait_all(bar_p(t, 1), j & 1);
        if (!ok) break;
        tc_fence_after();
        issue_pv(t, j, 1);
        // Stage j % kStages is free once both tiles' PV (and, earlier, S) read it.
        if (t == kTiles - 1) commit(bar_kvempty(j % kStages));
        if (j + 1 < n_kv) {
          if (t == 0) {
            ok = wait_all(bar_kvfull((j + 1) % kStages), ((j + 1) / kStages) & 1);
            if (!ok) break;
            tc_fence_after();
          }
          issue_s(t, j + 1);
        } else {
          commit(bar_o(t));
        }
      }
    }
  } else {
    // ---------------- softmax: warp -> (tile, lane quadrant), thread -> query row ----------------
    const int t = warp >> 2;
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    const uint32_t lanes = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + lanes + kTmemS + t * 128;
    const uint32_t t_o = tmem + lanes + kTmemO + t * 128;
    const float c = prm.scale_log2;
    float m_use = -INFINITY;  // running row max, log2 units, that P is taken against
    float l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      ok = wait_bar(bar_s(t), j & 1, abort_flag, prm.status);
      // tcgen05.ld/st below are warp-collective.
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sv[4][32];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) tmem_ld32(t_s + 32 * q4, sv[q4]);
      tmem_ld_wait(sv[0]);
      tmem_pin(sv[1]);
      tmem_pin(sv[2]);
      tmem_pin(sv[3]);
      const int valid = prm.seq_k - (j0 + j) * kBlockN;  // keys of this block that exist
      if (valid < kBlockN) {
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) mask_keys(sv[q4], 32 * q4, valid);
      }
      // p = 2^(s*c - m) in packed fp32x2 for keys [64h, 64h+64); kPolyPairs of
      // every 8 pairs take the FMA-pipe exp2.
      const float2 c2 = make_float2(c, c);
      float2 acc[2];
      uint32_t pk[32];
      auto exponentiate = [&](int h, float m) {
        const float2 nm2 = make_float2(-m, -m);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = 64 * h + 2 * i;
          const uint32_t* src = sv[key >> 5] + (key & 31);
          const float2 x =
              __ffma2_rn(make_float2(__uint_as_float(src[0]), __uint_as_float(src[1])), c2, nm2);
          float2 p;
          if ((i & 7) >= 8 - kPolyPairs) {
            p = exp2_poly(x);
          } else {
            p.x = ex2(x.x);
            p.y = ex2(x.y);
          }
          acc[i & 1] = __fadd2_rn(acc[i & 1], p);
          pk[i] = pack_bf16(p.x, p.y);
        }
      };
      // Row max over the 128 scores (eight independent 3-input max chains) and,
      // independent of it, the first half of P against the running max: the
      // scheduler interleaves the two, so the max costs no latency. The half is
      // redone in the rare case that the max moved by more than the threshold
      // (always at j = 0, where the running max is still -inf).
      float mx[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) {
        const uint32_t* r = sv[a >> 1] + (a & 1) * 16;
        float m = max3(__uint_as_float(r[0]), __uint_as_float(r[1]), __uint_as_float(r[2]));
#pragma unroll
        for (int k = 3; k < 15; k += 2) m = max3(m, __uint_as_float(r[k]), __uint_as_float(r[k + 1]));
        mx[a] = fmaxf(m, __uint_as_float(r[15]));
      }
      acc[0] = acc[1] = make_float2(0.f, 0.f);
      exponentiate(0, m_use);
      const float row_max = fmaxf(max3(mx[0], mx[1], mx[2]), max3(mx[3], max3(mx[4], mx[5], mx[6]), mx[7]));
      const float m_new = row_max * c;
      const bool need = m_new > m_use + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {
        const float m_next = need ? m_new : m_use;
        if (j > 0) {
          // PV_t(j-1) is complete: the S_t(j) commit covers every earlier MMA.
          const float alpha = ex2(m_use - m_next);  // 1 for rows that keep their max
          // 16 columns at a time: the row's 128 scores stay live in registers.
#pragma unroll 1
          for (int q8 = 0; q8 < 8; ++q8) {
            uint32_t o[16];
            tmem_ld16(t_o + 16 * q8, o);
            tmem_ld_wait16(o);
#pragma unroll
            for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st16(t_o + 16 * q8, o);
          }
          l_sum *= alpha;
        }
        m_use = m_next;
        // S columns [0, 64) are still intact: reload them rather than keep the
        // first half's scores live in registers across this rare branch.
        tmem_ld32(t_s, sv[0]);
        tmem_ld32(t_s + 32, sv[1]);
        tmem_ld_wait(sv[0]);
        tmem_pin(sv[1]);
        if (valid < kBlockN) {
          mask_keys(sv[0], 0, valid);
          mask_keys(sv[1], 32, valid);
        }
        acc[0] = acc[1] = make_float2(0.f, 0.f);
        exponentiate(0, m_use);
      }
      // P of keys [64h, 64h+64) -> S columns [32h, 32h+32), already read.
      tmem_st32(t_s, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar_p(t, 0));
      exponentiate(1, m_use);
      tmem_st32(t_s + 32, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(bar_p(t, 1));
      l_sum += (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
    }
    // ---------------- epilogue: O / l -> bf16 (or fp32 partials) ----------------
    if (ok) {
      ok = wait_bar(bar_o(t), 0, abort_flag, prm.status);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const int row = q_row0 + t * kBlockM + row_in_tile;
      const float inv_l = 1.f / l_sum;
      float* ws = split_slot >= 0
                      ? prm.ws + (int64_t)split_slot * kWsSlotFloats + t * kWsTileFloats
                      : nullptr;
      __nv_bfloat16* dst =
          (ws == nullptr && row < prm.seq_q) ? out_row(prm, batch, row, head) : nullptr;
#pragma unroll 1
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t o[32];
        tmem_ld32(t_o + 32 * q4, o);
        tmem_ld_wait(o);
        if (ws != nullptr) {
          // Partial result of a key range: unnormalised O and (running max, sum).
          float* o_row = ws + row_in_tile * kHeadDim + 32 * q4;
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4)
            *reinterpret_cast<float4*>(o_row + v4 * 4) =
                make_float4(__uint_as_float(o[v4 * 4 + 0]), __uint_as_float(o[v4 * 4 + 1]),
                            __uint_as_float(o[v4 * 4 + 2]), __uint_as_float(o[v4 * 4 + 3]));
        } else if (row < prm.seq_q) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            uint4 u;
            u.x = pack_bf16(__uint_as_float(o[v8 * 8 + 0]) * inv_l,
                            __uint_as_float(o[v8 * 8 + 1]) * inv_l);
            u.y = pack_bf16(__uint_as_float(o[v8 * 8 + 2]) * inv_l,
                            __uint_as_float(o[v8 * 8 + 3]) * inv_l);
            u.z = pack_bf16(__uint_as_float(o[v8 * 8 + 4]) * inv_l,
                            __uint_as_float(o[v8 * 8 + 5]) * inv_l);
            u.w = pack_bf16(__uint_as_float(o[v8 * 8 + 6]) * inv_l,
                            __uint_as_float(o[v8 * 8 + 7]) * inv_l);
            *reinterpret_cast<uint4*>(dst + 32 * q4 + v8 * 8) = u;
          }
        }
      }
      if (ws != nullptr) {
        float* ml = ws + kBlockM * kHeadDim + 2 * row_in_tile;
        ml[0] = m_use;
        ml[1] = l_sum;
      } else if (prm.route.world != 0) {
        __threadfence_system();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}


// Merges the key-range partials of the split units: one warp per query row,
// 4 head dims per lane. O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
__global__ void __launch_bounds__(256) attention_combine(const Params prm, int split_units) {
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  constexpr int kRowsPerUnit = kTiles * kBlockM;
  if (gw >= split_units * kRowsPerUnit) return;
  const int ui = gw / kRowsPerUnit;
  const int rr = gw - ui * kRowsPerUnit;
  const int t = rr / kBlockM;
  const int r_in_tile = rr - t * kBlockM;
  const int unit = prm.n_full + ui;
  const int qb = unit % prm.units_per_bh;
  const int bh = unit / prm.units_per_bh;
  const int head = bh % prm.heads;
  const int batch = bh / prm.heads;
  const int row = qb * kRowsPerUnit + rr;
  if (row >= prm.seq_q) return;
  auto tile_ws = [&](int split) {
    return prm.ws + (int64_t)(ui * prm.splits + split) * kWsSlotFloats + t * kWsTileFloats;
  };
  float m_max = -INFINITY;
  for (int sp = 0; sp < prm.splits; ++sp)
    m_max = fmaxf(m_max, tile_ws(sp)[kBlockM * kHeadDim + 2 * r_in_tile]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float l_tot = 0.f;
  for (int sp = 0; sp < prm.splits; ++sp) {
    const float* w = tile_ws(sp);
    const float scale = ex2(w[kBlockM * kHeadDim + 2 * r_in_tile] - m_max);
    l_tot += scale * w[kBlockM * kHeadDim + 2 * r_in_tile + 1];
    const float4 o = *reinterpret_cast<const float4*>(w + r_in_tile * kHeadDim + lane * 4);
    acc.x += scale * o.x;
    acc.y += scale * o.y;
    acc.z += scale * o.z;
    acc.w += scale * o.w;
  }
  const float inv = 1.f / l_tot;
  __nv_bfloat16* dst = out_row(prm, batch, row, head) + lane * 4;
  uint2 u;
  u.x = pack_bf16(acc.x * inv, acc.y * inv);
  u.y = pack_bf16(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(dst) = u;
  if (prm.route.world != 0) __threadfence_system();
}

// Work plan of one call: which units run whole and how the last, partial wave
// of units is split along the keys so that it fills the GPU.
struct Plan {
  int units_per_bh, units, n_full, splits, blocks_per_split, grid, split_units;
  int64_t ws_bytes;
};

Plan make_plan(int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads) {
  Plan pl{};
  pl.units_per_bh = (int)((seq_q + kTiles * kBlockM - 1) / (kTiles * kBlockM));
  pl.units = (int)(pl.units_per_bh * heads * batch);
  const int n_kv = (int)((seq_k + kBlockN - 1) / kBlockN);
  const int sms = num_sms();
  const int rem = pl.units % sms;
  pl.splits = 1;
  pl.blocks_per_split = n_kv;
  if (rem > 0 && 2 * rem <= sms && n_kv >= 2) {
    int want = sms / rem;
    if (want > 32) want = 32;
    if (want > n_kv) want = n_kv;
    pl.blocks_per_split = (n_kv + want - 1) / want;
    pl.splits = (n_kv + pl.blocks_per_split - 1) / pl.blocks_per_split;
  }
  if (pl.splits >= 2) {
    pl.split_units = rem;
    pl.n_full = pl.units - rem;
    pl.grid = pl.n_full + rem * pl.splits;
    pl.ws_bytes = (int64_t)rem * pl.splits * kWsSlotFloats * (int64_t)sizeof(float);
  } else {
    pl.splits = 1;
    pl.blocks_per_split = n_kv;
    pl.split_units = 0;
    pl.n_full = pl.units;
    pl.grid = pl.units;
    pl.ws_bytes = 0;
  }
  return pl;
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

// 4-D map over (head_dim, heads, rows, batch) with a (64, 1, 128, 1) box.
int make_map(CUtensorMap* map, const void* base, int64_t batch, int64_t seq, int64_t heads,
             int64_t bs, int64_t rs, int64_t hs, const char* name) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    set_error("h3b_attention: cuTensorMapEncodeTiled is unavailable");
    return H3B_ERR_CUDA;
  }
  // Size-1 dimensions never step their stride; give them a valid one.
  if (heads == 1) hs = kHeadDim;
  if (batch == 1) bs = rs * (seq > 0 ? seq : 1);
  cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)heads, (cuuint64_t)seq,
                        (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)hs * 2, (cuuint64_t)rs * 2, (cuuint64_t)bs * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)kBlockM, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "h3b_attention: tensor map for %s rejected (CUresult %d)", name,
             (int)r);
    set_error(buf);
    return H3B_ERR_CUDA;
  }
  return H3B_OK;
}

}  // namespace attn
}  // namespace h3b

namespace {

// h3b_attention with an optional output route (nullptr: the local `out`).
int attention_launch(void* out, const void* q, const void* k, const void* v, int64_t batch,
                     int64_t seq_q, int64_t seq_k, int64_t heads, int64_t head_dim,
                     int64_t q_batch_stride, int64_t q_row_stride, int64_t q_head_stride,
                     int64_t k_batch_stride, int64_t k_row_stride, int64_t k_head_stride,
                     int64_t v_batch_stride, int64_t v_row_stride, int64_t v_head_stride,
                     int64_t o_batch_stride, int64_t o_row_stride, int64_t o_head_stride,
                     float softmax_scale, void* workspace, int64_t workspace_bytes,
                     const h3b::attn::OutRoute* route, h3b_stream_t stream) {
  using namespace h3b::attn;
  H3B_REQUIRE(batch >= 0 && seq_q >= 0 && seq_k >= 0 && heads >= 0,
              "attention: negative shape");
  if (head_dim != kHeadDim) {
    h3b::set_error("h3b_attention: head_dim must be 128");
    return H3B_ERR_UNSUPPORTED;
  }
  if (batch == 0 || seq_q == 0 || heads == 0) return H3B_OK;
  H3B_REQUIRE(seq_k > 0, "attention: empty key sequence");
  H3B_REQUIRE(seq_q < (1LL << 31) && seq_k < (1LL << 31) &&
                  ((seq_q + 255) / 256) * heads * batch < (1LL << 31),
              "attention: shape exceeds launch limits");
  H3B_REQUIRE(h3b::aligned16(q) && h3b::aligned16(k) && h3b::aligned16(v) &&
                  (route != nullptr || h3b::aligned16(out)),
              "attention: q, k, v, out must be 16-byte aligned");
  const int64_t strides[12] = {q_batch_stride, q_row_stride, q_head_stride, k_batch_stride,
                               k_row_stride,   k_head_stride, v_batch_stride, v_row_stride,
                               v_head_stride,  o_batch_stride, o_row_stride, o_head_stride};
  for (int i = 0; i < (route != nullptr ? 9 : 12); ++i) {
    const bool unit = (i % 3 == 0 && batch == 1) || (i % 3 == 2 && heads == 1);
    H3B_REQUIRE(unit || (strides[i] % 8 == 0 && strides[i] > 0),
                "attention: strides must be positive multiples of 8 elements");
  }
  CUtensorMap qm, km, vm;
  int rc;
  if ((rc = make_map(&qm, q, batch, seq_q, heads, q_batch_stride, q_row_stride, q_head_stride,
                     "q")) != H3B_OK)
    return rc;
  if ((rc = make_map(&km, k, batch, seq_k, heads, k_batch_stride, k_row_stride, k_head_stride,
                     "k")) != H3B_OK)
    return rc;
  if ((rc = make_map(&vm, v, batch, seq_k, heads, v_batch_stride, v_row_stride, v_head_stride,
                     "v")) != H3B_OK)
    return rc;
  {
    // Set once per device and context (a function attribute belongs to the context).
    static h3b::ContextSlot attr_slots[h3b::kMaxDevices];
    cudaError_t e = cudaErrorInvalidDevice;
    if (h3b::context_cached(attr_slots, [&]() -> void* {
          e = cudaFuncSetAttribute(attention_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kSmemAlloc);
          return e == cudaSuccess ? reinterpret_cast<void*>(1) : nullptr;
        }) == nullptr) {
      h3b::set_error(std::string("h3b_attention: cannot reserve shared memory: ") +
                     cudaGetErrorString(e));
      return H3B_ERR_CUDA;
    }
  }
  Plan pl = make_plan(batch, seq_q, seq_k, heads);
  if (pl.ws_bytes > 0 && (workspace == nullptr || workspace_bytes < pl.ws_bytes ||
                          !h3b::aligned16(workspace))) {
    // No (or too small a) workspace: run every unit whole.
    pl.splits = 1;
    pl.split_units = 0;
    pl.n_full = pl.grid = pl.units;
    pl.blocks_per_split = (int)((seq_k + kBlockN - 1) / kBlockN);
    pl.ws_bytes = 0;
  }
  Params p;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.o_batch_stride = o_batch_stride;
  p.o_row_stride = o_row_stride;
  p.o_head_stride = o_head_stride;
  if (route != nullptr) {
    p.route = *route;
  } else {
    memset(&p.route, 0, sizeof(p.route));
  }
  p.seq_q = (int)seq_q;
  p.seq_k = (int)seq_k;
  p.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
  p.status = h3b::status_ptr();
  p.heads = (int)heads;
  p.units_per_bh = pl.units_per_bh;
  p.n_full = pl.n_full;
  p.splits = pl.splits;
  p.blocks_per_split = pl.blocks_per_split;
  p.ws = reinterpret_cast<float*>(workspace);
  attention_fwd<<<(unsigned)pl.grid, kThreads, kSmemAlloc, stream>>>(qm, km, vm, p);
  if (pl.split_units > 0) {
    int rc = h3b::check_launch("h3b_attention");
    if (rc != H3B_OK) return rc;
    const int warps = pl.split_units * kTiles * kBlockM;
    attention_combine<<<(unsigned)((warps + 7) / 8), 256, 0, stream>>>(p, pl.split_units);
  }
  return h3b::check_launch("h3b_attention");
}

}  // namespace

extern "C" int h3b_attention(void* out, const void* q, const void* k, const void* v,
                             int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads,
                             int64_t head_dim, int64_t q_batch_stride, int64_t q_row_stride,
                             int64_t q_head_stride, int64_t k_batch_stride,
                             int64_t k_row_stride, int64_t k_head_stride,
                             int64_t v_batch_stride, int64_t v_row_stride,
                             int64_t v_head_stride, int64_t o_batch_stride,
                             int64_t o_row_stride, int64_t o_head_stride, float softmax_scale,
                             void* workspace, int64_t workspace_bytes, h3b_stream_t stream) {
  return attention_launch(out, q, k, v, batch, seq_q, seq_k, heads, head_dim, q_batch_stride,
                          q_row_stride, q_head_stride, k_batch_stride, k_row_stride,
                          k_head_stride, v_batch_stride, v_row_stride, v_head_stride,
                          o_batch_stride, o_row_stride, o_head_stride, softmax_scale, workspace,
                          workspace_bytes, nullptr, stream);
}

extern "C" int h3b_attention_p2p(void* const* merged_ptrs, const int64_t* row_counts,
                                 int64_t world, int64_t rank, const void* qkv,
                                 int64_t heads_local, int64_t head_dim, float softmax_scale,
                                 void* workspace, int64_t workspace_bytes,
                                 h3b_stream_t stream) {
  using namespace h3b::attn;
  using h3b::kMaxPeers;
  H3B_REQUIRE(world >= 1 && world <= kMaxPeers, "attention_p2p: world size must be 1..%d",
              kMaxPeers);
  H3B_REQUIRE(rank >= 0 && rank < world, "attention_p2p: rank %lld outside world %lld",
              (long long)rank, (long long)world);
  H3B_REQUIRE(merged_ptrs != nullptr && row_counts != nullptr && qkv != nullptr,
              "attention_p2p: null argument");
  H3B_REQUIRE(heads_local > 0 && heads_local * world <= (1LL << 20),
              "attention_p2p: heads_local must be positive");
  if (head_dim != kHeadDim) {
    h3b::set_error("h3b_attention_p2p: head_dim must be 128");
    return H3B_ERR_UNSUPPORTED;
  }
  OutRoute route;
  memset(&route, 0, sizeof(route));
  for (int i = 0; i < world; ++i) {
    H3B_REQUIRE(row_counts[i] >= 0, "attention_p2p: negative row count");
    H3B_REQUIRE(merged_ptrs[i] != nullptr && h3b::aligned16(merged_ptrs[i]),
                "attention_p2p: merged buffer of rank %d is null or not 16-byte aligned", i);
    route.dst.p[i] = merged_ptrs[i];
    route.start[i + 1] = route.start[i] + row_counts[i];
  }
  for (int i = (int)world + 1; i <= kMaxPeers; ++i) route.start[i] = route.start[world];
  route.world = (int)world;
  route.head_base = (int)(rank * heads_local);
  route.heads_total = (int)(heads_local * world);
  const int64_t seq = route.start[world];
  if (seq == 0) return H3B_OK;
  // The packed receive buffer [S, hl, 3D]: q | k | v per head.
  const auto* base = static_cast<const __nv_bfloat16*>(qkv);
  const int64_t rs = heads_local * 3 * kHeadDim, hs = 3 * kHeadDim;
  return attention_launch(nullptr, base, base + kHeadDim, base + 2 * kHeadDim, 1, seq, seq,
                          heads_local, head_dim, 0, rs, hs, 0, rs, hs, 0, rs, hs, 0, 0, 0,
                          softmax_scale, workspace, workspace_bytes, &route, stream);
}

extern "C" int h3b_attention_workspace_size(int64_t batch, int64_t seq_q, int64_t seq_k,
                                            int64_t heads, int64_t head_dim,
                                            int64_t* bytes_out) {
  using namespace h3b::attn;
  H3B_REQUIRE(bytes_out != nullptr, "attention_workspace_size: null output pointer");
  H3B_REQUIRE(batch >= 0 && seq_q >= 0 && seq_k >= 0 && heads >= 0,
              "attention: negative shape");
  *bytes_out = 0;
  if (head_dim != kHeadDim || batch == 0 || seq_q == 0 || heads == 0 || seq_k == 0) return H3B_OK;
  *bytes_out = make_plan(batch, seq_q, seq_k, heads).ws_bytes;
  return H3B_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free entry point
// ---------------------------------------------------------------------------
//
// Some callers cannot hand this library scratch memory. A host runtime that
// reaches the kernels through the plain C ABI (an FFI binding inside a
// serving process) often has no device allocator of its own: the device
// memory belongs to another framework's pool, and calling cudaMalloc from the
// hot loop would step around that pool and can synchronise the whole device.
// h3b_attention_noalloc serves them: the split-tail workspace lives in the
// fixed device array below, so the call allocates nothing.
//
// The array is kNoAllocScratchBytes (20 MiB) on every GPU that loads this
// library, held until the process exits. It covers the largest split plan of a
// B200 (148 SMs x 130 KiB per split CTA); a shape whose plan needs more is
// rejected with H3B_ERR_VALUE. Every call on a device shares the one array and
// finds whatever the previous call left there. Nothing in it has to start at
// zero (each split CTA writes its whole slot before the combine kernel reads
// it), but two calls whose kernels overlap on the GPU race on it: run them on
// one stream, or order them.
constexpr int64_t kNoAllocScratchBytes = 20ll << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
h3b::ContextSlot g_noalloc_slot[h3b::kMaxDevices];

// Device address of g_noalloc_scratch on the current device. The first call on
// a device looks it up (cudaGetSymbolAddress, with that device current), and so
// does the first call after the device's context was re-created (cudaDeviceReset
// reloads the module, which can move the array); otherwise the cached address is
// used. In host code the array's name is only a host-side stand-in and must
// never reach a kernel.
int noalloc_scratch(void** out) {
  cudaError_t e = cudaErrorInvalidDevice;
  void* p = h3b::context_cached(g_noalloc_slot, [&]() -> void* {
    void* a = nullptr;
    e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
    return e == cudaSuccess ? a : nullptr;
  });
  if (p == nullptr) {
    h3b::set_error(std::string("h3b_attention_noalloc: cannot resolve the scratch array: ") +
                   cudaGetErrorString(e));
    return H3B_ERR_CUDA;
  }
  *out = p;
  return H3B_OK;
}
}  // namespace

extern "C" int h3b_attention_noalloc(void* out, const void* q, const void* k, const void* v,
                                     int64_t batch, int64_t seq_q, int64_t seq_k,
                                     int64_t heads, int64_t head_dim, int64_t q_batch_stride,
                                     int64_t q_row_stride, int64_t q_head_stride,
                                     int64_t k_batch_stride, int64_t k_row_stride,
                                     int64_t k_head_stride, int64_t v_batch_stride,
                                     int64_t v_row_stride, int64_t v_head_stride,
                                     int64_t o_batch_stride, int64_t o_row_stride,
                                     int64_t o_head_stride, float softmax_scale,
                                     h3b_stream_t stream) {
  int64_t need = 0;
  int rc = h3b_attention_workspace_size(batch, seq_q, seq_k, heads, head_dim, &need);
  if (rc != H3B_OK) return rc;
  if (need > kNoAllocScratchBytes) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "h3b_attention_noalloc: this shape needs %lld bytes of split workspace, more than "
             "the static maximum of %lld bytes; use h3b_attention with a caller workspace",
             (long long)need, (long long)kNoAllocScratchBytes);
    h3b::set_error(buf);
    return H3B_ERR_VALUE;
  }
  void* scratch = nullptr;
  if (need > 0 && (rc = noalloc_scratch(&scratch)) != H3B_OK) return rc;
  return h3b_attention(out, q, k, v, batch, seq_q, seq_k, heads, head_dim, q_batch_stride,
                       q_row_stride, q_head_stride, k_batch_stride, k_row_stride,
                       k_head_stride, v_batch_stride, v_row_stride, v_head_stride,
                       o_batch_stride, o_row_stride, o_head_stride, softmax_scale, scratch,
                       need > 0 ? kNoAllocScratchBytes : 0, stream);
}
