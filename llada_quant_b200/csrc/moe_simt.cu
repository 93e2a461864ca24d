// CUDA-core grouped expert GEMMs: the plain, obviously-correct implementation
// of the routed W4A16/W8A16 expert FFN.  It is the cross-check for the tcgen05
// kernels and the path for shapes those do not cover.  Numerics are the
// reference's: weights are bf16(q * s) exactly as dequantize_tensor
// (src/LLaDA_Quant/algorithms/symmetric.py:272-293), fp32 accumulation, and
// the epilogue rounding order of the external fused_moe kernel
// (INFERENCE_REPO_CHANGES.md:296-309 and :259-265).
#include "llq_common.cuh"

namespace llq {

namespace {

constexpr int kTileN = 64;     // output features per block
constexpr int kTileRows = 16;  // routed rows per pass
constexpr int kThreads = 256;  // 64 features x 4 row lanes

// 8 consecutive weights of one row as bf16-rounded floats
__device__ __forceinline__ void load_w8(const int8_t* __restrict__ q, int64_t row, int64_t K, int k,
                                        int bits, const float* __restrict__ srow, int group, float (&w)[8]) {
  const float s = srow[group > 0 ? k / group : 0];
  if (bits == 4) {
    const uint32_t packed = *reinterpret_cast<const uint32_t*>(q + row * (K >> 1) + (k >> 1));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int v = static_cast<int>(packed << (28 - 4 * i)) >> 28;
      w[i] = round_bf16(__fmul_rn(static_cast<float>(v), s));
    }
  } else {
    const uint2 packed = *reinterpret_cast<const uint2*>(q + row * K + k);
    const int8_t* b = reinterpret_cast<const int8_t*>(&packed);
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = round_bf16(__fmul_rn(static_cast<float>(b[i]), s));
  }
}

template <bool GEMM1>
__global__ void __launch_bounds__(kThreads) moe_gemm_simt_kernel(
    const __nv_bfloat16* __restrict__ a, const int32_t* __restrict__ offsets, int N_out, int K,
    int inter, const int8_t* __restrict__ q, const float* __restrict__ scale, int bits, int group,
    const int32_t* __restrict__ sorted_slots, const float* __restrict__ topk_w,
    __nv_bfloat16* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [kTileRows][K]
  const int e = blockIdx.y;
  const int n = blockIdx.x * kTileN + (threadIdx.x % kTileN);
  const int lane_row = threadIdx.x / kTileN;  // 0..3
  const int row0 = offsets[e], row1 = offsets[e + 1];
  const int groups = group > 0 ? K / group : 1;
  const int64_t rows_total = GEMM1 ? 2 * static_cast<int64_t>(inter) : N_out;
  const int64_t wrow_a = static_cast<int64_t>(e) * rows_total + n;          // gate / w2 row
  const int64_t wrow_b = wrow_a + inter;                                    // up row (GEMM1)
  const bool active = n < N_out;
  const float* srow_a = scale + wrow_a * groups;
  const float* srow_b = scale + wrow_b * groups;

  for (int r0 = row0; r0 < row1; r0 += kTileRows) {
    const int nr = row1 - r0 < kTileRows ? row1 - r0 : kTileRows;
    __syncthreads();
    const int vpr = K / 8;
    for (int i = threadIdx.x; i < kTileRows * vpr; i += kThreads) {
      const int r = i / vpr, v = i - r * vpr;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (r < nr) val = reinterpret_cast<const uint4*>(a + static_cast<int64_t>(r0 + r) * K)[v];
      reinterpret_cast<uint4*>(xs + static_cast<int64_t>(r) * K)[v] = val;
    }
    __syncthreads();
    if (!active) continue;
    float acc_a[kTileRows / 4], acc_b[kTileRows / 4];
#pragma unroll
    for (int j = 0; j < kTileRows / 4; ++j) acc_a[j] = acc_b[j] = 0.f;
    for (int k = 0; k < K; k += 8) {
      float wa[8], wb[8];
      load_w8(q, wrow_a, K, k, bits, srow_a, group, wa);
      if (GEMM1) load_w8(q, wrow_b, K, k, bits, srow_b, group, wb);
#pragma unroll
      for (int j = 0; j < kTileRows / 4; ++j) {
        const __nv_bfloat16* xr = xs + static_cast<int64_t>(lane_row + 4 * j) * K + k;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float xv = __bfloat162float(xr[i]);
          acc_a[j] = __fmaf_rn(xv, wa[i], acc_a[j]);
          if (GEMM1) acc_b[j] = __fmaf_rn(xv, wb[i], acc_b[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kTileRows / 4; ++j) {
      const int r = lane_row + 4 * j;
      if (r >= nr) continue;
      const int64_t p = r0 + r;
      if (GEMM1) {
        const float g = round_bf16(acc_a[j]);
        const float u = round_bf16(acc_b[j]);
        const float silu = round_bf16(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))));
        out[p * inter + n] = __float2bfloat16_rn(__fmul_rn(silu, u));
      } else {
        const int32_t slot = sorted_slots[p];
        out[static_cast<int64_t>(slot) * N_out + n] = __float2bfloat16_rn(__fmul_rn(acc_a[j], topk_w[slot]));
      }
    }
  }
}

int check_gemm_shape(int K, int group, int bits) {
  if (bits != 4 && bits != 8) return fail(LLQ_EINVAL, "bits must be 8 or 4, got %d", bits);
  if (K % 8 != 0) return fail(LLQ_EUNSUPPORTED, "K must be a multiple of 8, got %d", K);
  if (group > 0 && group % 8 != 0 && K % group == 0)
    return fail(LLQ_EUNSUPPORTED, "group size must be a multiple of 8, got %d", group);
  return LLQ_OK;
}

template <bool GEMM1>
int launch_simt(const void* a, const int32_t* offsets, int E, int N_out, int K, int inter,
                const int8_t* q, const float* scale, int bits, int group_size,
                const int32_t* sorted_slots, const float* topk_w, void* out, cudaStream_t st) {
  const int group = (group_size > 0 && K % group_size == 0) ? group_size : 0;
  int rc = check_gemm_shape(K, group, bits);
  if (rc) return rc;
  const size_t smem = static_cast<size_t>(kTileRows) * K * 2;
  if (smem > 200 * 1024) return fail(LLQ_EUNSUPPORTED, "K=%d too large for the SIMT GEMM", K);
  static std::atomic<uint64_t> attr{0};
  if (first_use_on_device(attr))
    cudaFuncSetAttribute(moe_gemm_simt_kernel<GEMM1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  dim3 grid((N_out + kTileN - 1) / kTileN, E);
  moe_gemm_simt_kernel<GEMM1><<<grid, kThreads, smem, st>>>(
      static_cast<const __nv_bfloat16*>(a), offsets, N_out, K, inter, q, scale, bits, group,
      sorted_slots, topk_w, static_cast<__nv_bfloat16*>(out));
  return check_launch("moe_gemm_simt_kernel");
}

}  // namespace

int gemm1_simt(const void* x_sorted, const int32_t* offsets, int E, int H, int I, const int8_t* qw1,
               const float* sw1, int bits, int group_size, void* h_sorted, cudaStream_t st) {
  return launch_simt<true>(x_sorted, offsets, E, I, H, I, qw1, sw1, bits, group_size, nullptr,
                           nullptr, h_sorted, st);
}

int gemm2_simt(const void* h_sorted, const int32_t* offsets, const int32_t* sorted_slots,
               const float* topk_w, int E, int H, int I, const int8_t* qw2, const float* sw2,
               int bits, int group_size, void* y_slots, cudaStream_t st) {
  return launch_simt<false>(h_sorted, offsets, E, H, I, I, qw2, sw2, bits, group_size,
                            sorted_slots, topk_w, y_slots, st);
}

}  // namespace llq
