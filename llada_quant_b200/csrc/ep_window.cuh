// Layout of an expert-parallel exchange window and the device-side flag helpers.
//
// Every rank of an expert-parallel group owns one window (one cudaMalloc'd
// block, shared with its peers through CUDA IPC handles); all windows have the
// same layout, so a kernel reaches field F of rank d's window at
// peers[d] + layout.F.  With R ranks and a capacity of `cap` (token, slot)
// entries per source rank:
//
//   sig   uint32 [5R + 8]   counts[R]   rows that rank s put in my region s
//                           dflag[R]    epoch of rank s's completed dispatch
//                           rflag[R]    epoch of rank d's completed return
//                           sendcnt[R]  my per-destination cursors (dispatch)
//                           spare[R]
//                           done[8]     last-block counters of my kernels
//   ids   int32 [R][cap]    expert id (local to me) of each received entry
//   wts   fp32  [R][cap]    its routed weight
//   rows  bf16  [R][cap][H] the received token rows, region s written by rank s
//   back  bf16  [R][cap][H] the returned expert outputs, region d written by rank d
//
// Rows only ever move by plain stores into a peer's window (no loads from a
// peer, no multicast).  A phase signals by a last-block pattern: every block
// fences its stores at system scope and counts itself done; the last one
// writes the flags with st.release.sys.  Waits poll with ld.acquire.sys under
// a time limit and record a code in g_device_error when it runs out.
#pragma once

#include "llq_common.cuh"

namespace llq {

struct EpLayout {
  size_t sig, ids, wts, rows, back, total;
  int R, cap, H;
};

__host__ __device__ inline size_t ep_align256(size_t v) { return (v + 255) / 256 * 256; }

__host__ __device__ inline EpLayout ep_layout(int R, int cap, int H) {
  EpLayout L{};
  L.R = R;
  L.cap = cap;
  L.H = H;
  size_t off = 0;
  L.sig = off;
  off = ep_align256(off + sizeof(uint32_t) * (5 * R + 8));
  L.ids = off;
  off = ep_align256(off + sizeof(int32_t) * static_cast<size_t>(R) * cap);
  L.wts = off;
  off = ep_align256(off + sizeof(float) * static_cast<size_t>(R) * cap);
  L.rows = off;
  off = ep_align256(off + static_cast<size_t>(R) * cap * H * 2);
  L.back = off;
  off = ep_align256(off + static_cast<size_t>(R) * cap * H * 2);
  L.total = off;
  return L;
}

enum EpSig { kEpCounts = 0, kEpDflag = 1, kEpRflag = 2, kEpSendcnt = 3 };

__host__ __device__ inline uint32_t* ep_sig(char* base, const EpLayout& L, int which) {
  return reinterpret_cast<uint32_t*>(base + L.sig) + which * L.R;
}
__host__ __device__ inline uint32_t* ep_done(char* base, const EpLayout& L, int i) {
  return reinterpret_cast<uint32_t*>(base + L.sig) + 5 * L.R + i;
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait until flags[0..R) have all reached `epoch` (wrap-safe), at most
// timeout_ns in total.  Returns false (and records `code`) if the time ran out.
__device__ inline bool ep_wait_flags(const uint32_t* flags, int R, uint32_t epoch, uint64_t timeout_ns,
                                     int code) {
  if (*reinterpret_cast<volatile int32_t*>(&g_device_error) == code) return false;  // already gave up
  const uint64_t t0 = global_ns();
  for (int s = 0; s < R; ++s) {
    unsigned ns = 32;
    while (static_cast<int32_t>(ld_acquire_sys(flags + s) - epoch) < 0) {
      if (global_ns() - t0 > timeout_ns) {
        atomicExch(&g_device_error, code);
        return false;
      }
      __nanosleep(ns);
      if (ns < 1024) ns <<= 1;
    }
  }
  return true;
}

constexpr int kMaxRanks = 64;

// Optional validity mask over the entries (expert-parallel receive windows):
// entry i is present iff (i % cap) < counts[i / cap]; before reading counts the
// single-block path waits for the R dispatch flags to reach `epoch`.
struct AlignMask {
  const uint32_t* counts;  // nullptr: every entry is present
  int cap;
  const uint32_t* flags;   // nullptr: no wait
  int R;
  uint32_t epoch;
  uint64_t timeout_ns;
  int32_t* clear;          // optional: zeroed by the alignment (the fused GEMMs' tile counters)
  int clear_n;
};

// Scatter target of the expert GEMM2 in expert-parallel mode: the output row of
// received entry `slot` (region s = slot / cap, position slot % cap) goes to
// rank s's back region, at my region there.
struct EpScatter {
  char* const* peers;  // device array of R window bases
  EpLayout L;
  int me;
  uint32_t epoch;
  uint32_t* done;  // my last-block counter for this phase
};

}  // namespace llq
