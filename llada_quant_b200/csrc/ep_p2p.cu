// Expert parallelism over NVLink peer memory: dispatch rows straight into the
// destination ranks' windows, run the local experts on what arrived, let the
// expert GEMM2 store each result straight back into its source rank's window,
// and combine once every rank's results are in.  No host synchronisation and
// no collective library on the data path: device flags carry the epochs.
//
// Protocol of one layer call (epoch e, every rank, stream order):
//   1. dispatch   each (token, slot) entry -> rank d = id / experts_per_rank,
//                 row + (local id, weight) stored at my region of d's window;
//                 the last block writes counts[me] and dflag[me] = e at every d
//   2. experts    wait for dflag[0..R) >= e; align the present entries by local
//                 expert; permute; GEMM1; GEMM2 stores into each source rank's
//                 back region; its last CTA writes rflag[me] = e at every rank
//   3. combine    wait for rflag[0..R) >= e; out[t] = sum over slots in order
// A window is reused by the next call safely: a rank's dispatch of e+1 follows
// its combine of e, which waited for every rank's GEMM2 of e -- the last reader
// of the receive regions that the dispatch of e+1 overwrites.
#include <cstring>

#include "llq_internal.cuh"

namespace llq {

namespace {

uint64_t g_timeout_ns = 5000000000ull;  // bounded cross-GPU waits: 5 s by default

constexpr int kDispatchThreads = 256;

// One warp per (token, slot) entry.
__global__ void __launch_bounds__(kDispatchThreads) ep_dispatch_kernel(
    const uint4* __restrict__ x, const int32_t* __restrict__ topk_ids, const float* __restrict__ topk_w,
    int64_t n, int k, int vpr, int experts_per_rank, char* const* __restrict__ peers, char* mine, EpLayout L,
    int me, uint32_t epoch, int32_t* __restrict__ inv_pos) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kDispatchThreads / 32);
  uint32_t* sendcnt = ep_sig(mine, L, kEpSendcnt);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * (kDispatchThreads / 32) + (threadIdx.x >> 5); i < n;
       i += warps) {
    const int32_t e = topk_ids[i];
    const int d = e >= 0 ? e / experts_per_rank : -1;
    int pos = 0;
    if (lane == 0) {
      if (d < 0 || d >= L.R) {
        atomicExch(&g_device_error, 2);
        pos = -1;
      } else {
        pos = static_cast<int>(atomicAdd(sendcnt + d, 1u));
        if (pos >= L.cap) {
          atomicExch(&g_device_error, 0x504);
          pos = -1;
        }
      }
    }
    pos = __shfl_sync(0xffffffffu, pos, 0);
    if (pos < 0) {
      if (lane == 0) inv_pos[i] = -1;
      continue;
    }
    char* peer = peers[d];
    const int64_t at = static_cast<int64_t>(me) * L.cap + pos;
    const uint4* src = x + (i / k) * vpr;
    uint4* dst = reinterpret_cast<uint4*>(peer + L.rows) + at * vpr;
    // all of a lane's loads of a 4 KiB slice before its stores: one round trip per slice
    constexpr int U = 8;
    for (int v0 = 0; v0 < vpr; v0 += 32 * U) {
      uint4 buf[U];
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int v = v0 + j * 32 + lane;
        if (v < vpr) buf[j] = __ldg(src + v);
      }
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int v = v0 + j * 32 + lane;
        if (v < vpr) dst[v] = buf[j];
      }
    }
    if (lane == 0) {
      reinterpret_cast<int32_t*>(peer + L.ids)[at] = e - d * experts_per_rank;
      reinterpret_cast<float*>(peer + L.wts)[at] = topk_w[i];
      inv_pos[i] = static_cast<int32_t>(static_cast<int64_t>(d) * L.cap + pos);
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(ep_done(mine, L, 0), 1u) == gridDim.x - 1) {
    __threadfence_system();
    for (int d = 0; d < L.R; ++d) ep_sig(peers[d], L, kEpCounts)[me] = atomicExch(sendcnt + d, 0u);
    __threadfence_system();
    for (int d = 0; d < L.R; ++d) st_release_sys(ep_sig(peers[d], L, kEpDflag) + me, epoch);
    atomicExch(ep_done(mine, L, 0), 0u);
  }
}

// out[t] = bf16(sum_j back[inv_pos[t*k + j]]) in fp32, slot order, once every
// rank has returned its rows.  Entries that were never sent (inv_pos < 0) add 0.
__global__ void ep_combine_wait_kernel(const uint4* back, const int32_t* __restrict__ inv_pos, int64_t T, int k,
                                       int vpr, uint4* __restrict__ out, const uint32_t* rflags, int R,
                                       uint32_t epoch, uint64_t timeout_ns) {
  if (threadIdx.x == 0) ep_wait_flags(rflags, R, epoch, timeout_ns, 0x503);
  __syncthreads();
  const int64_t total = T * vpr;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vpr;
    const int v = static_cast<int>(i - t * vpr);
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int64_t p = inv_pos[t * k + j];
      if (p < 0) continue;
      const uint4 yv = back[p * vpr + v];
      const __nv_bfloat16* yp = reinterpret_cast<const __nv_bfloat16*>(&yv);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = __fadd_rn(acc[q], __bfloat162float(yp[q]));
    }
    uint4 o;
    __nv_bfloat16* op = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) op[q] = __float2bfloat16_rn(acc[q]);
    out[i] = o;
  }
}

struct EpWorkspace {
  int32_t* offsets;
  int32_t* sorted_slots;
  void* align_ws;
  size_t align_bytes;
  void* x_sorted;
  void* h_sorted;
  int32_t* counters;  // the fused GEMMs' tile counters
  int n_counters;
  void* w1_bf16;      // windows that can hold prefill-sized calls: the shard's weights in bf16
  void* w2_bf16;
  size_t total;
};

EpWorkspace carve_ep(void* base, int R, int cap, int E, int H, int I) {
  EpWorkspace w{};
  const int64_t n = static_cast<int64_t>(R) * cap;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = ep_align256(off + bytes);
    return static_cast<char*>(base) + o;
  };
  w.offsets = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (E + 1)));
  w.sorted_slots = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * n));
  w.align_bytes = align_workspace_size(n, 1, E);
  w.align_ws = take(w.align_bytes);
  w.x_sorted = take(static_cast<size_t>(n) * H * 2 + 4096);
  w.h_sorted = take(static_cast<size_t>(n) * I * 2 + 4096);
  w.n_counters = gemm12_counter_slots(n, E);
  w.counters = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * w.n_counters));
  w.w1_bf16 = w.w2_bf16 = nullptr;
  if (n >= static_cast<int64_t>(E) * kPrefillRowsPerExpert) {
    w.w1_bf16 = take(static_cast<size_t>(E) * 2 * I * H * 2);
    w.w2_bf16 = take(static_cast<size_t>(E) * H * I * 2);
  }
  w.total = off;
  return w;
}

int check_window(int rank, int world, int cap, int H) {
  if (world < 1 || world > kMaxRanks) return fail(LLQ_EINVAL, "world size must be in [1, %d], got %d", kMaxRanks, world);
  if (rank < 0 || rank >= world) return fail(LLQ_EINVAL, "rank %d outside [0, %d)", rank, world);
  if (cap < 1) return fail(LLQ_EINVAL, "window capacity must be >= 1");
  if (H < 8 || H % 8 != 0) return fail(LLQ_EUNSUPPORTED, "hidden size must be a multiple of 8");
  if (static_cast<int64_t>(world) * cap > 0x7fffffff) return fail(LLQ_EINVAL, "window too large");
  return LLQ_OK;
}

unsigned grid_upto(int64_t blocks, int per_sm) {
  const int64_t lim = static_cast<int64_t>(num_sms()) * per_sm;
  if (blocks > lim) blocks = lim;
  if (blocks < 1) blocks = 1;
  return static_cast<unsigned>(blocks);
}

}  // namespace
}  // namespace llq

using namespace llq;

extern "C" {

size_t llq_ep_window_bytes(int world, int cap, int H) {
  if (world < 1 || cap < 1 || H < 1) return 0;
  return ep_layout(world, cap, H).total;
}

int llq_ep_set_timeout_ms(int ms) {
  if (ms < 1) return fail(LLQ_EINVAL, "timeout must be >= 1 ms");
  g_timeout_ns = static_cast<uint64_t>(ms) * 1000000ull;
  return LLQ_OK;
}

int llq_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr || bytes == 0) return fail(LLQ_EINVAL, "bad ipc_alloc arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(LLQ_ECUDA, "ipc window: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return LLQ_OK;
}

int llq_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

int llq_ipc_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return fail(LLQ_EINVAL, "bad ipc_open arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr = p;
  return LLQ_OK;
}

int llq_ipc_close(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return LLQ_OK;
}

int llq_ipc_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "cudaFree: %s", cudaGetErrorString(e));
  return LLQ_OK;
}

int llq_ep_dispatch(const void* x, const int32_t* topk_ids, const float* topk_w, int64_t T, int k, int H,
                    int experts_per_rank, void* window, void* const* peers, int rank, int world, int cap,
                    uint32_t epoch, int32_t* inv_pos, void* stream) {
  int rc = check_window(rank, world, cap, H);
  if (rc) return rc;
  if (T < 0 || k < 1 || experts_per_rank < 1) return fail(LLQ_EINVAL, "bad dispatch shape");
  if (T * k > cap) return fail(LLQ_EINVAL, "T*k = %lld exceeds the window capacity %d", (long long)(T * k), cap);
  if (window == nullptr || peers == nullptr) return fail(LLQ_EINVAL, "null window");
  const EpLayout L = ep_layout(world, cap, H);
  const int64_t n = T * k;
  const unsigned grid = grid_upto((n + kDispatchThreads / 32 - 1) / (kDispatchThreads / 32), 8);
  ep_dispatch_kernel<<<grid, kDispatchThreads, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(x), topk_ids, topk_w, n, k, H / 8, experts_per_rank,
      reinterpret_cast<char* const*>(peers), static_cast<char*>(window), L, rank, epoch, inv_pos);
  return check_launch("ep_dispatch_kernel");
}

size_t llq_ep_experts_workspace_size(int world, int cap, int E, int H, int I) {
  if (world < 1 || cap < 1 || E < 1) return 0;
  return carve_ep(nullptr, world, cap, E, H, I).total;
}

int llq_ep_experts(void* window, void* const* peers, int rank, int world, int cap, uint32_t epoch,
                   const int8_t* qw1, const float* sw1, const int8_t* qw2, const float* sw2, int E, int H,
                   int I, int bits, int group_size, int64_t rows_hint, void* workspace,
                   size_t workspace_bytes, int impl, void* stream) {
  int rc = check_window(rank, world, cap, H);
  if (rc) return rc;
  if (window == nullptr || peers == nullptr) return fail(LLQ_EINVAL, "null window");
  if (impl == LLQ_GEMM_SIMT)
    return fail(LLQ_EUNSUPPORTED, "the peer-memory expert path runs on the tcgen05 GEMMs only");
  const bool fast = impl == LLQ_GEMM_TCGEN05_FAST;
  if (fast && bits != 4) return fail(LLQ_EUNSUPPORTED, "fast dequantization is INT4 only");
  if (!tc_supported(E, I, H, bits, group_size, true) || !tc_supported(E, H, I, bits, group_size, false))
    return fail(LLQ_EUNSUPPORTED, "tcgen05 expert GEMMs do not cover E=%d H=%d I=%d bits=%d group=%d", E, H,
                I, bits, group_size);
  const EpWorkspace ws = carve_ep(workspace, world, cap, E, H, I);
  if (workspace == nullptr || workspace_bytes < ws.total)
    return fail(LLQ_ENOSPACE, "workspace needs %zu bytes, got %zu", ws.total, workspace_bytes);
  cudaStream_t st = as_stream(stream);
  char* mine = static_cast<char*>(window);
  const EpLayout L = ep_layout(world, cap, H);
  const int64_t n = static_cast<int64_t>(world) * cap;
  AlignMask m{};
  m.counts = ep_sig(mine, L, kEpCounts);
  m.cap = cap;
  m.flags = ep_sig(mine, L, kEpDflag);
  m.R = world;
  m.epoch = epoch;
  m.timeout_ns = g_timeout_ns;
  m.clear = ws.counters;
  m.clear_n = ws.n_counters;
  rc = align_impl_masked(reinterpret_cast<const int32_t*>(mine + L.ids), n, E, ws.offsets, ws.sorted_slots,
                         ws.align_ws, ws.align_bytes, st, m);
  if (rc) return rc;
  rc = permute_impl(mine + L.rows, n, H, 1, ws.sorted_slots, ws.x_sorted, st, fast ? 1 : 0, ws.offsets + E);
  if (rc) return rc;
  if (rows_hint < 0) rows_hint = n;
  EpScatter sc{};
  sc.peers = reinterpret_cast<char* const*>(peers);
  sc.L = L;
  sc.me = rank;
  sc.epoch = epoch;
  sc.done = ep_done(mine, L, 1);
  if (!fast && ws.w1_bf16 != nullptr && rows_hint >= static_cast<int64_t>(E) * kPrefillRowsPerExpert) {
    // prefill-sized call: the shard's weights dequantized once, bf16 GEMMs from shared memory
    rc = dequantize_impl(qw1, sw1, static_cast<int64_t>(E) * 2 * I, H, bits, group_size, bits == 4, ws.w1_bf16,
                         LLQ_BF16, st);
    if (rc) return rc;
    rc = dequantize_impl(qw2, sw2, static_cast<int64_t>(E) * H, I, bits, group_size, bits == 4, ws.w2_bf16,
                         LLQ_BF16, st);
    if (rc) return rc;
    return gemm12_fused_bf16_tc(ws.x_sorted, ws.offsets, ws.sorted_slots, reinterpret_cast<const float*>(mine + L.wts),
                                n, E, H, I, ws.w1_bf16, ws.w2_bf16, ws.h_sorted, nullptr, ws.counters, st, &sc);
  }
  if (!fast)  // GEMM1 and GEMM2 in one launch; GEMM2 rows go straight to the source ranks
    return gemm12_fused_tc(ws.x_sorted, ws.offsets, ws.sorted_slots, reinterpret_cast<const float*>(mine + L.wts), n,
                           E, H, I, qw1, sw1, qw2, sw2, bits, group_size, ws.h_sorted, nullptr, ws.counters, st,
                           rows_hint, &sc);
  rc = gemm1_tc(ws.x_sorted, ws.offsets, n, E, H, I, qw1, sw1, bits, group_size, ws.h_sorted, fast, st,
                rows_hint);
  if (rc) return rc;
  return gemm2_tc(ws.h_sorted, ws.offsets, ws.sorted_slots, reinterpret_cast<const float*>(mine + L.wts), n, E,
                  H, I, qw2, sw2, bits, group_size, nullptr, fast, st, rows_hint, &sc);
}

int llq_ep_combine_wait(void* window, int rank, int world, int cap, uint32_t epoch, const int32_t* inv_pos,
                        int64_t T, int k, int H, void* out, void* stream) {
  int rc = check_window(rank, world, cap, H);
  if (rc) return rc;
  if (window == nullptr) return fail(LLQ_EINVAL, "null window");
  if (T < 0 || k < 1) return fail(LLQ_EINVAL, "bad combine shape");
  char* mine = static_cast<char*>(window);
  const EpLayout L = ep_layout(world, cap, H);
  const int vpr = H / 8;
  const unsigned grid = grid_upto((T * vpr + 255) / 256, 32);
  ep_combine_wait_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4*>(mine + L.back), inv_pos, T, k, vpr, static_cast<uint4*>(out),
      ep_sig(mine, L, kEpRflag), world, epoch, g_timeout_ns);
  return check_launch("ep_combine_wait_kernel");
}

}  // extern "C"
