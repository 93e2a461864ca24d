// extern "C" boundary of libllada_quant_cuda.so (declared in include/llada_quant.h).
#include <cstdarg>
#include <cstring>

#include "llq_common.cuh"
#include "llq_internal.cuh"

namespace llq {

__device__ int32_t g_device_error = 0;

namespace {
thread_local char t_error[512] = {0};
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
  return code;
}

const char* last_error() { return t_error; }

constexpr int KC_STEP = 128;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct MoeWorkspace {
  int32_t* offsets;
  int32_t* sorted_slots;
  void* align_ws;
  size_t align_bytes;
  void* x_sorted;
  void* h_sorted;
  void* y_slots;
  int32_t* tile_done;
  int tile_done_n;
  void* w1_bf16;  // prefill-sized calls: the layer's weights dequantized once (else null)
  void* w2_bf16;
  size_t total;
};

// prefill-sized call: enough routed rows per expert that every weight meets many
// token tiles, so dequantizing the weights once and running bf16 GEMMs is cheaper
bool prefill_call(int64_t T, int k, int E) { return T * k >= static_cast<int64_t>(E) * kPrefillRowsPerExpert; }

MoeWorkspace carve(void* base, int64_t T, int k, int E, int H, int I) {
  MoeWorkspace w{};
  const int64_t n = T * k;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return static_cast<char*>(base) + o;
  };
  w.offsets = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (E + 1)));
  w.sorted_slots = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * (n > 0 ? n : 1)));
  w.align_bytes = align_workspace_size(T, k, E);
  w.align_ws = take(w.align_bytes);
  w.x_sorted = take(static_cast<size_t>(n) * H * 2 + 4096);
  w.h_sorted = take(static_cast<size_t>(n) * I * 2 + 4096);
  w.y_slots = take(static_cast<size_t>(n) * H * 2 + 4096);
  w.tile_done_n = gemm12_counter_slots(n, E);
  w.tile_done = reinterpret_cast<int32_t*>(take(sizeof(int32_t) * w.tile_done_n));
  w.w1_bf16 = w.w2_bf16 = nullptr;
  if (prefill_call(T, k, E)) {
    w.w1_bf16 = take(static_cast<size_t>(E) * 2 * I * H * 2);
    w.w2_bf16 = take(static_cast<size_t>(E) * H * I * 2);
  }
  w.total = off;
  return w;
}

int pick_impl(int impl, int E, int N_out, int K, int bits, int group_size, bool gemm1) {
  if (impl == LLQ_GEMM_SIMT) return LLQ_GEMM_SIMT;
  const bool tc = tc_supported(E, N_out, K, bits, group_size, gemm1);
  if (impl == LLQ_GEMM_TCGEN05) return tc ? LLQ_GEMM_TCGEN05 : -1;
  if (impl == LLQ_GEMM_TCGEN05_FAST) return (tc && bits == 4) ? LLQ_GEMM_TCGEN05_FAST : -1;
  if (impl != LLQ_GEMM_AUTO) return -1;
  return tc ? LLQ_GEMM_TCGEN05 : LLQ_GEMM_SIMT;
}

}  // namespace llq

using namespace llq;

extern "C" {

int llq_version(void) { return 100; }

const char* llq_last_error(void) { return llq::last_error(); }

int llq_quantize_pack(const void* w, int w_dtype, int64_t rows, int64_t K, int bits, int group_size,
                      int search, int grid, double max_shrink, int scale_round, int pack, int8_t* q,
                      float* scale, void* stream) {
  return quantize_impl(w, w_dtype, rows, K, bits, group_size, search, grid, max_shrink, scale_round,
                       pack, q, scale, nullptr, as_stream(stream));
}

int llq_search_errors(const void* w, int w_dtype, int64_t rows, int64_t K, int bits, int group_size,
                      int grid, double max_shrink, float* errors, void* stream) {
  if (errors == nullptr) return fail(LLQ_EINVAL, "null errors pointer");
  return quantize_impl(w, w_dtype, rows, K, bits, group_size, LLQ_SEARCH_MSE, grid, max_shrink,
                       LLQ_F32, 0, nullptr, nullptr, errors, as_stream(stream));
}

int llq_dequantize(const int8_t* q, const float* scale, int64_t rows, int64_t K, int bits,
                   int group_size, int packed, void* out, int out_dtype, void* stream) {
  return dequantize_impl(q, scale, rows, K, bits, group_size, packed, out, out_dtype, as_stream(stream));
}

int llq_pack_int4(const int8_t* values, int64_t n, int8_t* packed, int32_t* range_error, void* stream) {
  if (range_error == nullptr) return fail(LLQ_EINVAL, "range_error must point to a device int32");
  return pack_int4_impl(values, n, packed, range_error, as_stream(stream));
}

int llq_unpack_int4(const int8_t* packed, int64_t n, int8_t* values, void* stream) {
  return unpack_int4_impl(packed, n, values, as_stream(stream));
}

int llq_route(const void* x, const void* gate_w, int64_t T, int H, int E, int k, const float* bias,
              int renormalize, void* logits, float* topk_w, int32_t* topk_ids, void* stream) {
  return route_impl(x, gate_w, T, H, E, k, bias, renormalize, logits, topk_w, topk_ids, as_stream(stream));
}

int llq_route_topk(const void* logits, int logits_dtype, int64_t T, int E, int k, const float* bias,
                   int renormalize, float* topk_w, int32_t* topk_ids, void* stream) {
  return route_topk_impl(logits, logits_dtype, T, E, k, bias, renormalize, topk_w, topk_ids,
                         as_stream(stream));
}

size_t llq_align_workspace_size(int64_t T, int k, int E) { return align_workspace_size(T, k, E); }

int llq_moe_align(const int32_t* topk_ids, int64_t T, int k, int E, int32_t* expert_offsets,
                  int32_t* sorted_slots, void* workspace, size_t workspace_bytes, void* stream) {
  return align_impl(topk_ids, T, k, E, expert_offsets, sorted_slots, workspace, workspace_bytes,
                    as_stream(stream));
}

int llq_moe_permute(const void* x, int64_t T, int H, int k, const int32_t* sorted_slots, int kperm,
                    void* x_sorted, void* stream) {
  return permute_impl(x, T, H, k, sorted_slots, x_sorted, as_stream(stream), kperm);
}

int llq_ep_pack(const void* x, const int32_t* topk_ids, const float* topk_w, int64_t T, int k, int H,
                int experts_per_rank, const int32_t* sorted_slots, void* send_rows, int32_t* local_ids,
                float* weights, int32_t* inv_pos, void* stream) {
  return ep_pack_impl(x, topk_ids, topk_w, T, k, H, experts_per_rank, sorted_slots, send_rows, local_ids, weights,
                      inv_pos, as_stream(stream));
}

int llq_ep_combine(const void* back_rows, const int32_t* inv_pos, int64_t T, int k, int H, void* out,
                   void* stream) {
  return ep_combine_impl(back_rows, inv_pos, T, k, H, out, as_stream(stream));
}

int llq_moe_combine(const void* y_slots, int64_t T, int k, int H, void* out, void* stream) {
  return combine_impl(y_slots, T, k, H, out, as_stream(stream));
}

int llq_moe_gemm1(const void* x_sorted, const int32_t* expert_offsets, int64_t n_rows, int E, int H,
                  int I, const int8_t* qw1, const float* sw1, int bits, int group_size,
                  void* h_sorted, int impl, void* stream) {
  const int which = pick_impl(impl, E, I, H, bits, group_size, true);
  if (which < 0) return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM1 does not cover this shape");
  if (which == LLQ_GEMM_TCGEN05 || which == LLQ_GEMM_TCGEN05_FAST)
    return gemm1_tc(x_sorted, expert_offsets, n_rows, E, H, I, qw1, sw1, bits, group_size,
                    h_sorted, which == LLQ_GEMM_TCGEN05_FAST, as_stream(stream));
  return gemm1_simt(x_sorted, expert_offsets, E, H, I, qw1, sw1, bits, group_size, h_sorted,
                    as_stream(stream));
}

int llq_moe_gemm2(const void* h_sorted, const int32_t* expert_offsets, const int32_t* sorted_slots,
                  const float* topk_w, int64_t n_rows, int E, int H, int I, const int8_t* qw2,
                  const float* sw2, int bits, int group_size, void* y_slots, int impl, void* stream) {
  const int which = pick_impl(impl, E, H, I, bits, group_size, false);
  if (which < 0) return fail(LLQ_EUNSUPPORTED, "tcgen05 GEMM2 does not cover this shape");
  if (which == LLQ_GEMM_TCGEN05 || which == LLQ_GEMM_TCGEN05_FAST)
    return gemm2_tc(h_sorted, expert_offsets, sorted_slots, topk_w, n_rows, E, H, I, qw2, sw2,
                    bits, group_size, y_slots, which == LLQ_GEMM_TCGEN05_FAST, as_stream(stream));
  return gemm2_simt(h_sorted, expert_offsets, sorted_slots, topk_w, E, H, I, qw2, sw2, bits,
                    group_size, y_slots, as_stream(stream));
}

size_t llq_quant_linear_workspace_size(int64_t M, int K, int N) {
  if (M <= 0 || K < KC_STEP || N < 1) return 0;
  const int ks = dense_ksplit(M, K, N);
  return ks > 1 ? static_cast<size_t>(ks) * M * N * 4 : 0;
}

int llq_quant_linear(const void* x, int64_t M, int K, int N, const int8_t* qweight, const float* scale, int bits,
                     int group_size, void* out, void* workspace, size_t workspace_bytes, int impl, void* stream) {
  if (M < 0 || K < 1 || N < 1) return fail(LLQ_EINVAL, "bad shape M=%lld K=%d N=%d", (long long)M, K, N);
  if (bits != 4 && bits != 8) return fail(LLQ_EUNSUPPORTED, "bits must be 8 or 4, got %d", bits);
  if (bits == 4 && K % 2 != 0) return fail(LLQ_EINVAL, "int4 packing needs an even last dimension");
  if (M == 0) return LLQ_OK;
  if (impl != LLQ_GEMM_AUTO && impl != LLQ_GEMM_TCGEN05)
    return fail(LLQ_EUNSUPPORTED, "the dense W%dA16 linear runs the exact tcgen05 kernel only", bits);
  if (M > 0x7fffffff) return fail(LLQ_EINVAL, "too many rows");
  return dense_linear_tc(x, M, K, N, qweight, scale, bits, group_size, out, workspace, workspace_bytes,
                         as_stream(stream));
}

size_t llq_moe_gemm12_counters(int64_t n_rows, int E) {
  if (n_rows < 0 || E < 1) return 0;
  return static_cast<size_t>(gemm12_counter_slots(n_rows, E));
}

int llq_moe_gemm12(const void* x_sorted, const int32_t* expert_offsets, const int32_t* sorted_slots,
                   const float* topk_w, int64_t n_rows, int E, int H, int I, const int8_t* qw1, const float* sw1,
                   const int8_t* qw2, const float* sw2, int bits, int group_size, void* h_sorted, void* y_slots,
                   int32_t* counters, void* stream) {
  if (n_rows < 0 || E < 1 || H < 1 || I < 1) return fail(LLQ_EINVAL, "bad shape");
  if (counters == nullptr) return fail(LLQ_EINVAL, "null counters");
  if (n_rows == 0) return LLQ_OK;
  if (pick_impl(LLQ_GEMM_TCGEN05, E, I, H, bits, group_size, true) < 0 ||
      pick_impl(LLQ_GEMM_TCGEN05, E, H, I, bits, group_size, false) < 0)
    return fail(LLQ_EUNSUPPORTED, "the fused expert GEMMs need the tcgen05 shapes (K %% 128 == 0, K <= 2048, "
                                  "I %% 128 == 0, H %% 256 == 0, group %% 128 == 0)");
  return gemm12_fused_tc(x_sorted, expert_offsets, sorted_slots, topk_w, n_rows, E, H, I, qw1, sw1, qw2, sw2, bits,
                         group_size, h_sorted, y_slots, counters, as_stream(stream));
}

size_t llq_moe_workspace_size(int64_t T, int k, int E, int H, int I) {
  return carve(nullptr, T, k, E, H, I).total;
}

}  // extern "C"

namespace llq {
namespace {

// the layer after the alignment: permute, expert GEMMs, combine
int experts_after_align(const MoeWorkspace& ws, const void* x, const int8_t* qw1, const float* sw1,
                        const int8_t* qw2, const float* sw2, const float* topk_w, int64_t T, int E, int H, int I,
                        int k, int bits, int group_size, void* out, int impl, cudaStream_t st) {
  const int64_t n = T * k;
  int rc;
  if (impl == LLQ_GEMM_TCGEN05_FAST) {
    rc = permute_impl(x, T, H, k, ws.sorted_slots, ws.x_sorted, st, 1);
    if (rc) return rc;
    rc = gemm12_fused_tc(ws.x_sorted, ws.offsets, ws.sorted_slots, topk_w, n, E, H, I, qw1, sw1, qw2, sw2, bits,
                         group_size, ws.h_sorted, ws.y_slots, ws.tile_done, st, -1, nullptr, true);
    if (rc) return rc;
    return combine_impl(ws.y_slots, T, k, H, out, st);
  }
  rc = permute_impl(x, T, H, k, ws.sorted_slots, ws.x_sorted, st, 0);
  if (rc) return rc;
  if (ws.w1_bf16 != nullptr && pick_impl(impl, E, I, H, bits, group_size, true) == LLQ_GEMM_TCGEN05 &&
      pick_impl(impl, E, H, I, bits, group_size, false) == LLQ_GEMM_TCGEN05) {
    // the weights are bit-identical to dequantize_tensor's, so are the products
    rc = dequantize_impl(qw1, sw1, static_cast<int64_t>(E) * 2 * I, H, bits, group_size, bits == 4, ws.w1_bf16,
                         LLQ_BF16, st);
    if (rc) return rc;
    rc = dequantize_impl(qw2, sw2, static_cast<int64_t>(E) * H, I, bits, group_size, bits == 4, ws.w2_bf16,
                         LLQ_BF16, st);
    if (rc) return rc;
    rc = gemm12_fused_bf16_tc(ws.x_sorted, ws.offsets, ws.sorted_slots, topk_w, n, E, H, I, ws.w1_bf16, ws.w2_bf16,
                              ws.h_sorted, ws.y_slots, ws.tile_done, st);
    if (rc) return rc;
    return combine_impl(ws.y_slots, T, k, H, out, st);
  }
  if (pick_impl(impl, E, I, H, bits, group_size, true) == LLQ_GEMM_TCGEN05 &&
      pick_impl(impl, E, H, I, bits, group_size, false) == LLQ_GEMM_TCGEN05) {
    rc = gemm12_fused_tc(ws.x_sorted, ws.offsets, ws.sorted_slots, topk_w, n, E, H, I, qw1, sw1, qw2, sw2, bits,
                         group_size, ws.h_sorted, ws.y_slots, ws.tile_done, st);
    if (rc) return rc;
    return combine_impl(ws.y_slots, T, k, H, out, st);
  }
  void* stream = st;
  rc = llq_moe_gemm1(ws.x_sorted, ws.offsets, n, E, H, I, qw1, sw1, bits, group_size, ws.h_sorted, impl, stream);
  if (rc) return rc;
  rc = llq_moe_gemm2(ws.h_sorted, ws.offsets, ws.sorted_slots, topk_w, n, E, H, I, qw2, sw2, bits, group_size,
                     ws.y_slots, impl, stream);
  if (rc) return rc;
  return combine_impl(ws.y_slots, T, k, H, out, st);
}

int check_fast(int impl, int E, int H, int I, int bits, int group_size) {
  if (impl == LLQ_GEMM_TCGEN05_FAST && (pick_impl(impl, E, I, H, bits, group_size, true) < 0 ||
                                        pick_impl(impl, E, H, I, bits, group_size, false) < 0))
    return fail(LLQ_EUNSUPPORTED, "LLQ_GEMM_TCGEN05_FAST does not cover this shape (INT4, K <= 2048, "
                                  "I %% 128 == 0, H %% 256 == 0, group %% 128 == 0)");
  return LLQ_OK;
}

// the alignment of a layer call: offsets and sorted slots; zeroes the GEMM tile counters
int align_layer(const MoeWorkspace& ws, const int32_t* topk_ids, int64_t n, int E, cudaStream_t st) {
  AlignMask am{};
  am.clear = ws.tile_done;
  am.clear_n = ws.tile_done_n;
  return align_impl_masked(topk_ids, n, E, ws.offsets, ws.sorted_slots, ws.align_ws, ws.align_bytes, st, am);
}

}  // namespace
}  // namespace llq

extern "C" {

int llq_fused_moe_packed(const void* x, const int8_t* qw1, const float* sw1, const int8_t* qw2,
                         const float* sw2, const float* topk_w, const int32_t* topk_ids, int64_t T,
                         int E, int H, int I, int k, int bits, int group_size, void* out,
                         void* workspace, size_t workspace_bytes, int impl, void* stream) {
  if (T < 0 || E < 1 || H < 1 || I < 1 || k < 1 || k > E)
    return fail(LLQ_EINVAL, "bad shape T=%lld E=%d H=%d I=%d k=%d", (long long)T, E, H, I, k);
  if (T == 0) return LLQ_OK;
  MoeWorkspace ws = carve(workspace, T, k, E, H, I);
  if (workspace == nullptr || workspace_bytes < ws.total)
    return fail(LLQ_ENOSPACE, "workspace needs %zu bytes, got %zu", ws.total, workspace_bytes);
  int rc = check_fast(impl, E, H, I, bits, group_size);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  rc = align_layer(ws, topk_ids, T * k, E, st);
  if (rc) return rc;
  return experts_after_align(ws, x, qw1, sw1, qw2, sw2, topk_w, T, E, H, I, k, bits, group_size, out, impl, st);
}

int llq_moe_block_packed(const void* x, const void* gate_w, const float* bias, int renormalize, int64_t T, int E,
                         int H, int I, int k, const int8_t* qw1, const float* sw1, const int8_t* qw2,
                         const float* sw2, int bits, int group_size, void* logits, float* topk_w,
                         int32_t* topk_ids, void* out, void* workspace, size_t workspace_bytes, int impl,
                         void* stream) {
  if (T < 0 || E < 1 || H < 1 || I < 1 || k < 1 || k > E)
    return fail(LLQ_EINVAL, "bad shape T=%lld E=%d H=%d I=%d k=%d", (long long)T, E, H, I, k);
  if (T == 0) return LLQ_OK;
  if (topk_w == nullptr || topk_ids == nullptr) return fail(LLQ_EINVAL, "null topk_w / topk_ids");
  MoeWorkspace ws = carve(workspace, T, k, E, H, I);
  if (workspace == nullptr || workspace_bytes < ws.total)
    return fail(LLQ_ENOSPACE, "workspace needs %zu bytes, got %zu", ws.total, workspace_bytes);
  int rc = check_fast(impl, E, H, I, bits, group_size);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  rc = route_impl(x, gate_w, T, H, E, k, bias, renormalize, logits, topk_w, topk_ids, st);
  if (rc) return rc;
  rc = align_layer(ws, topk_ids, T * k, E, st);
  if (rc) return rc;
  return experts_after_align(ws, x, qw1, sw1, qw2, sw2, topk_w, T, E, H, I, k, bits, group_size, out, impl, st);
}

int llq_device_error(int32_t* code) {
  if (code == nullptr) return fail(LLQ_EINVAL, "null code pointer");
  cudaError_t e = cudaMemcpyFromSymbol(code, g_device_error, sizeof(int32_t));
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "reading the device error word: %s", cudaGetErrorString(e));
  return LLQ_OK;
}

int llq_clear_device_error(void) {
  const int32_t zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int32_t));
  if (e != cudaSuccess) return fail(LLQ_ECUDA, "clearing the device error word: %s", cudaGetErrorString(e));
  return LLQ_OK;
}

}  // extern "C"
