// Internal entry points shared between the library's translation units.
#pragma once

#include "ep_window.cuh"

namespace llq {

int quantize_impl(const void*, int, int64_t, int64_t, int, int, int, int, double, int, int, int8_t*,
                  float*, float*, cudaStream_t);
int dequantize_impl(const int8_t*, const float*, int64_t, int64_t, int, int, int, void*, int,
                    cudaStream_t);
int pack_int4_impl(const int8_t*, int64_t, int8_t*, int32_t*, cudaStream_t);
int unpack_int4_impl(const int8_t*, int64_t, int8_t*, cudaStream_t);
int route_impl(const void*, const void*, int64_t, int, int, int, const float*, int, void*, float*,
               int32_t*, cudaStream_t);
int route_topk_impl(const void*, int, int64_t, int, int, const float*, int, float*, int32_t*,
                    cudaStream_t);
size_t align_workspace_size(int64_t, int, int);
int align_impl(const int32_t*, int64_t, int, int, int32_t*, int32_t*, void*, size_t, cudaStream_t);
int permute_impl(const void*, int64_t, int, int, const int32_t*, void*, cudaStream_t, int,
                 const int32_t* n_dev = nullptr);
int combine_impl(const void*, int64_t, int, int, void*, cudaStream_t);
int ep_pack_impl(const void*, const int32_t*, const float*, int64_t, int, int, int, const int32_t*, void*, int32_t*,
                 float*, int32_t*, cudaStream_t);
int ep_combine_impl(const void*, const int32_t*, int64_t, int, int, void*, cudaStream_t);
int gemm1_simt(const void*, const int32_t*, int, int, int, const int8_t*, const float*, int, int,
               void*, cudaStream_t);
int gemm2_simt(const void*, const int32_t*, const int32_t*, const float*, int, int, int,
               const int8_t*, const float*, int, int, void*, cudaStream_t);
int gemm1_tc(const void*, const int32_t*, int64_t, int, int, int, const int8_t*, const float*, int,
             int, void*, bool, cudaStream_t, int64_t rows_hint = -1);
int gemm2_tc(const void*, const int32_t*, const int32_t*, const float*, int64_t, int, int, int,
             const int8_t*, const float*, int, int, void*, bool, cudaStream_t, int64_t rows_hint = -1,
             const EpScatter* ep = nullptr);
bool tc_supported(int E, int N_out, int K, int bits, int group_size, bool gemm1);
// implementation an LLQ_GEMM_* request resolves to for one expert GEMM, or -1
int pick_impl(int impl, int E, int N_out, int K, int bits, int group_size, bool gemm1);

int dense_ksplit(int64_t M, int K, int N);
int gemm12_counter_slots(int64_t n_rows, int E);
int gemm12_fused_tc(const void* x_sorted, const int32_t* offsets, const int32_t* sorted_slots, const float* topk_w,
                    int64_t n_rows, int E, int H, int I, const int8_t* qw1, const float* sw1, const int8_t* qw2,
                    const float* sw2, int bits, int group_size, void* h_sorted, void* y_slots, int* tile_done,
                    cudaStream_t st, int64_t rows_hint = -1, const EpScatter* ep = nullptr,
                    bool fast = false);
int gemm12_fused_bf16_tc(const void* x_sorted, const int32_t* offsets, const int32_t* sorted_slots,
                         const float* topk_w, int64_t n_rows, int E, int H, int I, const void* w1, const void* w2,
                         void* h_sorted, void* y_slots, int* tile_done, cudaStream_t st,
                         const EpScatter* ep = nullptr);
// routed rows per expert from which a layer dequantizes its weights once and runs bf16 GEMMs
constexpr int64_t kPrefillRowsPerExpert = 512;
int dense_linear_tc(const void* x, int64_t M, int K, int N, const int8_t* q, const float* scale, int bits,
                    int group_size, void* out, void* workspace, size_t ws_bytes, cudaStream_t st);
int align_impl_masked(const int32_t*, int64_t, int, int32_t*, int32_t*, void*, size_t, cudaStream_t,
                      const AlignMask&);

}  // namespace llq
