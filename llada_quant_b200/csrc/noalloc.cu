// llq_fused_moe_packed_noalloc: the whole routed MoE layer without any device
// allocation by the caller or by the library.
//
// Some callers cannot hand the library a workspace: a plugin loaded into a host
// framework that owns the device allocator and exposes none of it to plugins,
// or a serving runtime that reserves all device memory at start-up and forbids
// allocation (and the device-wide synchronization cudaMalloc/cudaFree bring)
// afterwards.  For them this variant keeps its scratch in one file-scope
// device array of fixed size, so it needs no allocation at all.
//
// Scratch: g_noalloc_scratch, kNoAllocBytes (about 12 MiB), resident on every
// GPU that loads the library until the process exits.  Limits: T*k <= 2048
// routed rows, H <= 2048, I <= 1024, E <= 256 (the LLaDA-MoE-7B-A1B decode
// shape: 256 tokens x top-8).  Larger calls are rejected with LLQ_EINVAL.
//
// The first call on a device resolves the array's device address there
// (cudaGetSymbolAddress, with that device current) and caches it; make that
// first call before any stream capture.  Every call reuses the same array and
// finds the previous call's contents in it: nothing in it needs to start at
// zero (every byte a call reads was written earlier in the same call), but two
// calls whose executions overlap on the GPU -- on different streams, or from
// different host threads -- race on it and corrupt each other's results.
#include <mutex>

#include "llq_internal.cuh"

namespace llq {

namespace {

constexpr int64_t kNoAllocMaxRows = 2048;  // T * k
constexpr int kNoAllocMaxHidden = 2048;    // H
constexpr int kNoAllocMaxInter = 1024;     // I
constexpr int kNoAllocMaxExperts = 256;    // E

constexpr size_t kOffOffsets = 0;                                              // int32 [E+1]
constexpr size_t kOffSlots = 4096;                                             // int32 [rows]
constexpr size_t kOffAlign = kOffSlots + kNoAllocMaxRows * 4;                  // align counts
constexpr size_t kAlignBytes = 8192;
constexpr size_t kOffActs = kOffAlign + kAlignBytes;                           // bf16 [rows, H]: x_sorted, then y_slots
constexpr size_t kOffInter = kOffActs + kNoAllocMaxRows * kNoAllocMaxHidden * 2;  // bf16 [rows, I]
constexpr size_t kNoAllocBytes = kOffInter + kNoAllocMaxRows * kNoAllocMaxInter * 2;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (set up once per device).
int scratch_on_current_device(unsigned char** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(LLQ_EUNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(LLQ_ECUDA, "cudaGetSymbolAddress(g_noalloc_scratch): %s", cudaGetErrorString(e));
    g_scratch_ptr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_ptr[dev]);
  return LLQ_OK;
}

}  // namespace
}  // namespace llq

using namespace llq;

extern "C" {

int llq_moe_gemm1(const void*, const int32_t*, int64_t, int, int, int, const int8_t*, const float*, int, int,
                  void*, int, void*);
int llq_moe_gemm2(const void*, const int32_t*, const int32_t*, const float*, int64_t, int, int, int,
                  const int8_t*, const float*, int, int, void*, int, void*);

int llq_fused_moe_packed_noalloc(const void* x, const int8_t* qw1, const float* sw1, const int8_t* qw2,
                                 const float* sw2, const float* topk_w, const int32_t* topk_ids, int64_t T,
                                 int E, int H, int I, int k, int bits, int group_size, void* out, int impl,
                                 void* stream) {
  if (T < 0 || E < 1 || H < 1 || I < 1 || k < 1 || k > E)
    return fail(LLQ_EINVAL, "bad shape T=%lld E=%d H=%d I=%d k=%d", (long long)T, E, H, I, k);
  const int64_t rows = T * k;
  if (rows > kNoAllocMaxRows || H > kNoAllocMaxHidden || I > kNoAllocMaxInter || E > kNoAllocMaxExperts)
    return fail(LLQ_EINVAL,
                "llq_fused_moe_packed_noalloc: T*k=%lld H=%d I=%d E=%d exceeds its fixed scratch "
                "(T*k <= %lld, H <= %d, I <= %d, E <= %d); use llq_fused_moe_packed with a workspace",
                (long long)rows, H, I, E, (long long)kNoAllocMaxRows, kNoAllocMaxHidden, kNoAllocMaxInter,
                kNoAllocMaxExperts);
  if (align_workspace_size(T, k, E) > kAlignBytes)
    return fail(LLQ_EINVAL, "llq_fused_moe_packed_noalloc: alignment scratch too small");
  // the fast GEMM1 expects its token rows in the K-interleaved order its code
  // expansion produces, exactly as in llq_fused_moe_packed
  const bool fast = impl == LLQ_GEMM_TCGEN05_FAST;
  if (fast && (pick_impl(impl, E, I, H, bits, group_size, true) < 0 ||
               pick_impl(impl, E, H, I, bits, group_size, false) < 0))
    return fail(LLQ_EUNSUPPORTED, "LLQ_GEMM_TCGEN05_FAST does not cover this shape (INT4, K <= 2048, "
                                  "I %% 128 == 0, H %% 256 == 0, group %% 128 == 0)");
  if (T == 0) return LLQ_OK;
  unsigned char* base = nullptr;
  int rc = scratch_on_current_device(&base);
  if (rc) return rc;
  int32_t* offsets = reinterpret_cast<int32_t*>(base + kOffOffsets);
  int32_t* slots = reinterpret_cast<int32_t*>(base + kOffSlots);
  void* align_ws = base + kOffAlign;
  void* acts = base + kOffActs;    // x_sorted for GEMM1, then y_slots from GEMM2
  void* inter = base + kOffInter;  // h_sorted
  cudaStream_t st = as_stream(stream);
  rc = align_impl(topk_ids, T, k, E, offsets, slots, align_ws, kAlignBytes, st);
  if (rc) return rc;
  rc = permute_impl(x, T, H, k, slots, acts, st, fast ? 1 : 0);
  if (rc) return rc;
  rc = llq_moe_gemm1(acts, offsets, rows, E, H, I, qw1, sw1, bits, group_size, inter, impl, stream);
  if (rc) return rc;
  rc = llq_moe_gemm2(inter, offsets, slots, topk_w, rows, E, H, I, qw2, sw2, bits, group_size, acts, impl,
                     stream);
  if (rc) return rc;
  return combine_impl(acts, T, k, H, out, st);
}

}  // extern "C"
