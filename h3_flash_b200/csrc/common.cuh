// Shared helpers for the libh3b.so kernels: error plumbing, bf16 packing and
// 128-bit vector access. sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/h3b.h"

namespace h3b {

// Per-host-thread error string returned by h3b_last_error().
void set_error(const std::string& msg);
void clear_error();

// Returns H3B_OK or records the pending launch error and returns H3B_ERR_CUDA.
int check_launch(const char* what);

// Device address of this device's status word (bit flags documented in
// h3b.h), or nullptr if it cannot be resolved. Defined in abi.cu.
unsigned int* status_ptr();

// The calling thread's current CUDA context (the driver's handle), or nullptr.
// Per-device caches of module addresses and function attributes are keyed on
// it: cudaDeviceReset (or a released and re-created primary context) reloads
// the module, so a device ordinal alone does not identify a valid entry.
void* current_context();

// One per-device slot that remembers in which context it was filled. Readers
// and writers may race (concurrent first calls from several host threads);
// every field is atomic and filling a slot twice is harmless.
struct ContextSlot {
  std::atomic<void*> ctx{nullptr};
  std::atomic<void*> value{nullptr};
};
constexpr int kMaxDevices = 64;

// Runs fill() (which returns the slot's value, or nullptr on failure) when the
// slot for the current device was not filled in the current context. Returns
// the value, or nullptr if there is no usable device or fill() failed.
template <class Fill>
void* context_cached(ContextSlot (&slots)[kMaxDevices], Fill fill) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  void* ctx = current_context();
  ContextSlot& slot = slots[dev];
  if (ctx != nullptr && slot.ctx.load(std::memory_order_acquire) == ctx)
    return slot.value.load(std::memory_order_acquire);
  void* v = fill();
  if (v == nullptr) return nullptr;
  slot.value.store(v, std::memory_order_release);
  slot.ctx.store(ctx, std::memory_order_release);
  return v;
}

enum : unsigned int { kStatusAttentionTimeout = 1u };

#define H3B_REQUIRE(cond, ...)                                   \
  do {                                                           \
    if (!(cond)) {                                               \
      char _h3b_buf[512];                                        \
      snprintf(_h3b_buf, sizeof(_h3b_buf), __VA_ARGS__);         \
      ::h3b::set_error(_h3b_buf);                                \
      return H3B_ERR_VALUE;                                      \
    }                                                            \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- bf16 <-> fp32 ---------------------------------------------------------

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Round two fp32 values to nearest-even bf16 and pack (lo in bits 0..15).
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Device pointers of one buffer on every rank of a peer-mapped group (this
// rank's own entry is its local pointer). Passed by value as a kernel argument.
constexpr int kMaxPeers = 16;
struct PeerPtrs {
  void* p[kMaxPeers];
};
// p[i] for a runtime i without spilling the parameter array to local memory.
__device__ __forceinline__ void* peer_at(const PeerPtrs& pp, int i) {
  void* r = pp.p[0];
#pragma unroll
  for (int j = 1; j < kMaxPeers; ++j)
    if (i == j) r = pp.p[j];
  return r;
}

struct f8 {
  float v[8];
};

__device__ __forceinline__ f8 unpack8(uint4 u) {
  f8 r;
  r.v[0] = bf16lo(u.x); r.v[1] = bf16hi(u.x);
  r.v[2] = bf16lo(u.y); r.v[3] = bf16hi(u.y);
  r.v[4] = bf16lo(u.z); r.v[5] = bf16hi(u.z);
  r.v[6] = bf16lo(u.w); r.v[7] = bf16hi(u.w);
  return r;
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 u;
  u.x = pack_bf16(v[0], v[1]);
  u.y = pack_bf16(v[2], v[3]);
  u.z = pack_bf16(v[4], v[5]);
  u.w = pack_bf16(v[6], v[7]);
  return u;
}

// Streaming 128-bit accesses for data touched exactly once.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
// 32-byte (256-bit, sm_100) accesses: fewer, larger memory transactions. Used
// by the scatter whose stores cross NVLink to a peer's memory (+15% measured over
// 16-byte stores there; no gain in the pack, whose 32-byte pairs need a shuffle).
struct Chunk32 {
  uint4 lo, hi;
};
__device__ __forceinline__ Chunk32 ld_stream32(const void* p) {
  Chunk32 r;
  asm volatile("ld.global.cs.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r.lo.x), "=r"(r.lo.y), "=r"(r.lo.z), "=r"(r.lo.w), "=r"(r.hi.x),
                 "=r"(r.hi.y), "=r"(r.hi.z), "=r"(r.hi.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st32(void* p, const Chunk32& v) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v.lo.x),
               "r"(v.lo.y), "r"(v.lo.z), "r"(v.lo.w), "r"(v.hi.x), "r"(v.hi.y), "r"(v.hi.z),
               "r"(v.hi.w)
               : "memory");
}
inline bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

// Cached (L1/L2) read for small tables reused across rows.
__device__ __forceinline__ uint4 ld_cached(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

// ---- activations (fp32 in, fp32 out; MUFU ex2 / rcp) ---------------------

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcpf(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// silu(g) = g * sigmoid(g) = g / (1 + 2^(-g log2 e)): two MUFU ops, relative
// error a few fp32 ulps (results below 2^-126 flush to zero).
__device__ __forceinline__ float silu(float g) {
  return g * rcpf(1.f + ex2f(g * -1.4426950408889634f));
}

// gelu_tanh(x) = 0.5 x (1 + tanh(u)) = x * sigmoid(2u), u = sqrt(2/pi)(x + 0.044715 x^3),
// i.e. x / (1 + 2^(x (c1 + c2 x^2))) with c1 = -2 sqrt(2/pi) log2(e), c2 = c1 * 0.044715.
// The sigmoid form has no cancellation for negative x; two MUFU ops per element.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float c1 = -2.f * 0.7978845608028654f * 1.4426950408889634f;
  const float c2 = c1 * 0.044715f;
  const float e = ex2f(x * fmaf(c2, x * x, c1));
  return x * rcpf(1.f + e);
}

}  // namespace h3b
