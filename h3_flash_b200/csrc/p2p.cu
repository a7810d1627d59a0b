// Packed-Ulysses exchange over NVLink peer memory.
//
// With every rank's exchange buffers mapped into every process (CUDA IPC:
// plain peer loads and stores), the two all-to-alls of a
// packed-Ulysses attention call become stores issued by the kernels that
// produce the data:
//
//   h3b_qknorm_rope_pack_p2p (rope_pack.cu): QK-norm + RoPE + pack, each head
//       row stored into the receive buffer [S_total, hl, 3D] of the rank that
//       owns the head, at its global row (the QKV all-to-all).
//   h3b_scatter_heads_p2p: the attention output [S_total, hl, D] of this rank's
//       heads, each row stored into its owner's merged buffer [r_owner, H, D]
//       at head offset rank*hl (the output all-to-all and the head merge).
//   h3b_peer_barrier: every rank raises its slot in every peer's flag array and
//       waits, bounded, for all peers' slots in its own.
//
// One call runs pack_p2p, barrier, attention, scatter_p2p, barrier on one
// stream. Two barriers per call make single buffers safe: a rank writes a
// peer's receive buffer only after the peer has passed the previous call's
// second barrier, which it reaches after its attention read that buffer, and
// it writes a peer's merged buffer only after the peer has passed this call's
// first barrier, which it reaches after its previous output projection read it.
//
// The barrier's epoch is a counter in the rank's own flag array that the
// kernel advances itself, so the sequence can be captured in a CUDA graph.
//
// Semantics: src/h3_flash/runtime/parallel/packed_ulysses.py:85-128 and
// src/h3_flash/runtime/parallel/relayout.py:97-159.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "common.cuh"

namespace h3b {
namespace p2p {

struct RowOffsets {
  int64_t off[kMaxPeers + 1];
};

// A peer that has not arrived after this long is reported, not waited for.
constexpr unsigned long long kBarrierLimitNs = 10ull * 1000 * 1000 * 1000;
constexpr unsigned int kStatusPeerBarrierTimeout = 2u;
constexpr int kScatterThreads = 256;
constexpr int kScatterUnroll = 4;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Width in bytes of the chunks the scatter moves per thread: 32 (the 256-bit
// sm_100 loads/stores, fewer and larger remote writes) when the row width and
// the buffers allow it, else 16.
#ifndef H3B_SCATTER_BYTES
#define H3B_SCATTER_BYTES 32
#endif

template <int kBytes>
struct ChunkIO;
template <>
struct ChunkIO<16> {
  using T = uint4;
  static __device__ __forceinline__ T load(const void* p) { return ld_stream(p); }
  static __device__ __forceinline__ void store(void* p, const T& v) {
    *reinterpret_cast<uint4*>(p) = v;
  }
};
template <>
struct ChunkIO<32> {
  using T = Chunk32;
  static __device__ __forceinline__ T load(const void* p) { return ld_stream32(p); }
  static __device__ __forceinline__ void store(void* p, const T& v) { st32(p, v); }
};

// kBytes-wide chunks c of the [S_total, hl*D] output: chunk c of global row `row`
// goes to merged[owner][(row - off[owner]) * W + rank][c - row*inner].
template <int kBytes>
__global__ void __launch_bounds__(kScatterThreads) scatter_heads_kernel(
    PeerPtrs merged, RowOffsets offs, const __nv_bfloat16* __restrict__ out, int world,
    int rank, int64_t total_chunks, int64_t inner) {
  using IO = ChunkIO<kBytes>;
  constexpr int kElems = kBytes / 2;
  const int64_t base = (int64_t)blockIdx.x * (kScatterThreads * kScatterUnroll) + threadIdx.x;
  typename IO::T val[kScatterUnroll];
#pragma unroll
  for (int u = 0; u < kScatterUnroll; ++u) {
    const int64_t c = base + u * kScatterThreads;
    if (c < total_chunks) val[u] = IO::load(out + c * kElems);
  }
#pragma unroll
  for (int u = 0; u < kScatterUnroll; ++u) {
    const int64_t c = base + u * kScatterThreads;
    if (c < total_chunks) {
      const int64_t row = c / inner;
      const int64_t col = c - row * inner;
      // Owner = last rank whose first row is <= row (offsets never decrease).
      int owner = 0;
      int64_t first = 0;
#pragma unroll
      for (int j = 1; j < kMaxPeers; ++j)
        if (j < world && row >= offs.off[j]) owner = j, first = offs.off[j];
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peer_at(merged, owner)) +
                           (((row - first) * world + rank) * inner + col) * kElems;
      IO::store(dst, val[u]);
    }
  }
  __threadfence_system();
}

// flags.p[w] is rank w's flag array: slots [0, kMaxPeers) hold the epoch each
// peer last arrived with, slot kMaxPeers this rank's own epoch counter.
__global__ void peer_barrier_kernel(PeerPtrs flags, int world, int rank, unsigned int* status) {
  __shared__ unsigned int s_epoch;
  unsigned int* mine = reinterpret_cast<unsigned int*>(peer_at(flags, rank));
  if (threadIdx.x == 0) {
    s_epoch = mine[kMaxPeers] + 1u;
    mine[kMaxPeers] = s_epoch;
  }
  __syncthreads();
  const unsigned int epoch = s_epoch;
  const int w = threadIdx.x;
  if (w >= world) return;
  unsigned int* remote = reinterpret_cast<unsigned int*>(peer_at(flags, w)) + rank;
  asm volatile("fence.sc.sys;" ::: "memory");
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(remote), "r"(epoch) : "memory");
  const unsigned int* slot = mine + w;
  const unsigned long long t0 = globaltimer();
  for (unsigned int i = 0;; ++i) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(slot) : "memory");
    if ((int)(v - epoch) >= 0) break;
    if ((i & 63u) == 63u) {
      if (globaltimer() - t0 > kBarrierLimitNs) {
        atomicOr(status, kStatusPeerBarrierTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
}

int fill_ptrs(PeerPtrs& dst, void* const* src, int64_t world, const char* what) {
  H3B_REQUIRE(world >= 1 && world <= kMaxPeers, "%s: world size must be 1..%d", what, kMaxPeers);
  H3B_REQUIRE(src != nullptr, "%s: null pointer array", what);
  for (int i = 0; i < kMaxPeers; ++i) dst.p[i] = i < world ? src[i] : nullptr;
  for (int i = 0; i < world; ++i)
    H3B_REQUIRE(dst.p[i] != nullptr && aligned16(dst.p[i]),
                "%s: buffer of rank %d is null or not 16-byte aligned", what, i);
  return H3B_OK;
}

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

// A peer allocation can hold several exported buffers (allocators carve many
// tensors out of one cudaMalloc), but a process may map an IPC handle only
// once: mappings are shared per handle and reference-counted.
struct Mapping {
  void* base;
  int refs;
};
std::mutex g_ipc_mutex;
std::map<std::string, Mapping> g_ipc_maps;

int cuda_fail(cudaError_t e, const char* what) {
  char buf[256];
  snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
  set_error(buf);
  return H3B_ERR_CUDA;
}

}  // namespace p2p
}  // namespace h3b

using namespace h3b;
using namespace h3b::p2p;

extern "C" int h3b_scatter_heads_p2p(void* const* merged_ptrs, const int64_t* row_counts,
                                     const void* out, int64_t world, int64_t rank,
                                     int64_t heads_local, int64_t head_dim,
                                     h3b_stream_t stream) {
  PeerPtrs ptrs;
  int rc = fill_ptrs(ptrs, merged_ptrs, world, "scatter_heads_p2p");
  if (rc != H3B_OK) return rc;
  H3B_REQUIRE(rank >= 0 && rank < world, "scatter_heads_p2p: rank %lld outside world %lld",
              (long long)rank, (long long)world);
  H3B_REQUIRE(row_counts != nullptr, "scatter_heads_p2p: null row counts");
  H3B_REQUIRE(heads_local > 0 && head_dim > 0 && (heads_local * head_dim) % 8 == 0,
              "scatter_heads_p2p: heads_local*head_dim must be a positive multiple of 8");
  RowOffsets offs{};
  for (int i = 0; i < world; ++i) {
    H3B_REQUIRE(row_counts[i] >= 0, "scatter_heads_p2p: negative row count");
    offs.off[i + 1] = offs.off[i] + row_counts[i];
  }
  for (int i = (int)world + 1; i <= kMaxPeers; ++i) offs.off[i] = offs.off[world];
  const int64_t width = heads_local * head_dim;  // elements of one row of this rank's heads
  if (offs.off[world] == 0) return H3B_OK;
  H3B_REQUIRE(aligned16(out), "scatter_heads_p2p: out must be 16-byte aligned");
  bool wide = H3B_SCATTER_BYTES == 32 && width % 16 == 0 && aligned32(out);
  for (int i = 0; i < world && wide; ++i) wide = aligned32(ptrs.p[i]);
  const int64_t per_block = kScatterThreads * kScatterUnroll;
  if (wide) {
    const int64_t inner = width / 16, total_chunks = offs.off[world] * inner;
    scatter_heads_kernel<32><<<(unsigned)((total_chunks + per_block - 1) / per_block),
                               kScatterThreads, 0, stream>>>(
        ptrs, offs, (const __nv_bfloat16*)out, (int)world, (int)rank, total_chunks, inner);
  } else {
    const int64_t inner = width / 8, total_chunks = offs.off[world] * inner;
    scatter_heads_kernel<16><<<(unsigned)((total_chunks + per_block - 1) / per_block),
                               kScatterThreads, 0, stream>>>(
        ptrs, offs, (const __nv_bfloat16*)out, (int)world, (int)rank, total_chunks, inner);
  }
  return check_launch("h3b_scatter_heads_p2p");
}

extern "C" int h3b_peer_barrier(void* const* flag_ptrs, int64_t world, int64_t rank,
                                h3b_stream_t stream) {
  PeerPtrs ptrs;
  int rc = fill_ptrs(ptrs, flag_ptrs, world, "peer_barrier");
  if (rc != H3B_OK) return rc;
  H3B_REQUIRE(rank >= 0 && rank < world, "peer_barrier: rank %lld outside world %lld",
              (long long)rank, (long long)world);
  unsigned int* status = status_ptr();
  if (status == nullptr) return H3B_ERR_CUDA;
  peer_barrier_kernel<<<1, 32, 0, stream>>>(ptrs, (int)world, (int)rank, status);
  return check_launch("h3b_peer_barrier");
}

extern "C" int64_t h3b_peer_flags_bytes(void) {
  return (int64_t)(kMaxPeers + 1) * (int64_t)sizeof(unsigned int);
}

extern "C" int h3b_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
  H3B_REQUIRE(ptr != nullptr && handle != nullptr && offset != nullptr,
              "ipc_handle: null argument");
  auto range = address_range_fn();
  if (range == nullptr) {
    set_error("ipc_handle: cuMemGetAddressRange is unavailable");
    return H3B_ERR_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  CUresult r = range(&base, &size, (CUdeviceptr)ptr);
  if (r != CUDA_SUCCESS) {
    char buf[128];
    snprintf(buf, sizeof(buf), "ipc_handle: pointer is not device memory (CUresult %d)", (int)r);
    set_error(buf);
    return H3B_ERR_VALUE;
  }
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, (void*)base);
  if (e != cudaSuccess) return cuda_fail(e, "ipc_handle");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)((CUdeviceptr)ptr - base);
  return H3B_OK;
}

extern "C" int h3b_ipc_open(const void* handle, int64_t offset, void** ptr) {
  H3B_REQUIRE(handle != nullptr && ptr != nullptr && offset >= 0, "ipc_open: bad argument");
  const std::string key(static_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
  std::lock_guard<std::mutex> lock(g_ipc_mutex);
  auto it = g_ipc_maps.find(key);
  if (it == g_ipc_maps.end()) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "ipc_open");
    it = g_ipc_maps.emplace(key, Mapping{base, 0}).first;
  }
  it->second.refs += 1;
  *ptr = static_cast<char*>(it->second.base) + offset;
  return H3B_OK;
}

extern "C" int h3b_ipc_close(void* ptr, int64_t offset) {
  H3B_REQUIRE(ptr != nullptr && offset >= 0, "ipc_close: bad argument");
  void* base = static_cast<char*>(ptr) - offset;
  std::lock_guard<std::mutex> lock(g_ipc_mutex);
  for (auto it = g_ipc_maps.begin(); it != g_ipc_maps.end(); ++it) {
    if (it->second.base != base) continue;
    if (--it->second.refs > 0) return H3B_OK;
    g_ipc_maps.erase(it);
    cudaError_t e = cudaIpcCloseMemHandle(base);
    if (e != cudaSuccess) return cuda_fail(e, "ipc_close");
    return H3B_OK;
  }
  set_error("ipc_close: pointer was not opened by h3b_ipc_open");
  return H3B_ERR_VALUE;
}
