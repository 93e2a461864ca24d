/*
 * llada_quant.h -- C ABI of libllada_quant_cuda.so, the B200 (sm_100a) kernels
 * of LLaDA_Quant's quantized MoE expert path.
 *
 * Conventions
 *   - Plain pointers to DEVICE memory, sizes in elements, a cudaStream_t passed
 *     as void* (NULL = legacy default stream).  Every call is stream-ordered and
 *     asynchronous; none synchronizes the host.
 *   - The caller allocates every input, output and workspace
 *     (llq_moe_workspace_size says how much); the library never frees caller
 *     memory.
 *   - Return value: LLQ_OK (0) or an error code; llq_last_error() gives the
 *     message of the last failing call on the calling thread.  No C++ exception
 *     crosses this boundary.
 *   - Weights use the frozen LLaDA_Quant packed layout: q int8 [rows, K/2]
 *     (INT4, element 2i in the low nibble, two's complement) or [rows, K]
 *     (INT8); scale float32 [rows, K/group] (one scale per row when the group
 *     does not divide K, group == -1 in LLaDA_Quant's terms).
 *
 * Each entry point names the reference interface it replaces, by path within
 * the LLaDA_Quant project.
 */
#ifndef LLADA_QUANT_H
#define LLADA_QUANT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum llq_status {
  LLQ_OK = 0,
  LLQ_EINVAL = 1,       /* bad shape, pointer, alignment or argument */
  LLQ_EUNSUPPORTED = 2, /* valid but not implemented (bits, group, dtype) */
  LLQ_ECUDA = 3,        /* a CUDA launch or runtime call failed */
  LLQ_ETIMEOUT = 4,     /* a bounded device-side wait gave up */
  LLQ_ENOSPACE = 5      /* workspace too small */
};

enum llq_dtype { LLQ_F32 = 0, LLQ_F16 = 1, LLQ_BF16 = 2 };

enum llq_scale_search { LLQ_SEARCH_AMAX = 0, LLQ_SEARCH_MSE = 1 };

/*
 * Expert GEMM implementation.  AUTO = TCGEN05 where it covers the shape, else
 * SIMT.  TCGEN05 and SIMT use weights bit-identical to dequantize_tensor.
 * TCGEN05_FAST (INT4, whole-layer calls only) feeds the integer codes to the
 * tensor cores and applies each fp32 group scale to the group's fp32 partial
 * sum: W = q * s without the per-weight bf16 rounding.
 */
enum llq_gemm_impl {
  LLQ_GEMM_AUTO = 0,
  LLQ_GEMM_TCGEN05 = 1,
  LLQ_GEMM_SIMT = 2,
  LLQ_GEMM_TCGEN05_FAST = 3
};

/* Library version (major*10000 + minor*100 + patch). */
int llq_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* llq_last_error(void);

/* ------------------------------------------------------------------------ */
/* Quantize and pack.                                                        */
/* ------------------------------------------------------------------------ */

/*
 * Symmetric groupwise quantization of w [rows, K] along K, bit-exact with
 * quantize_tensor() (src/LLaDA_Quant/algorithms/symmetric.py:207-269) and,
 * for search == LLQ_SEARCH_MSE, search_group_scale() (:122-204) with the
 * given grid and max_shrink.  group_size == -1, or a group that does not
 * divide K, gives one scale per row (the fallback of _as_groups, :85-90).
 * scale_round rounds the chosen scale to that dtype before it is used and
 * stored (QuantConfig.scale_dtype): LLQ_F32 = keep.
 * pack != 0 with bits == 4 writes two values per byte (pack_int4, :296-313);
 * otherwise q holds one int8 per value.
 */
int llq_quantize_pack(const void* w, int w_dtype, int64_t rows, int64_t K, int bits,
                      int group_size, int search, int grid, double max_shrink,
                      int scale_round, int pack, int8_t* q, float* scale, void* stream);

/*
 * Per-group squared error of each MSE candidate (diagnostics for the
 * reduction-order analysis of search_group_scale, symmetric.py:188-202):
 * errors [rows * groups, grid] float32.
 */
int llq_search_errors(const void* w, int w_dtype, int64_t rows, int64_t K, int bits,
                      int group_size, int grid, double max_shrink, float* errors,
                      void* stream);

/*
 * w ~= q * scale, fp32 arithmetic then one rounding to out_dtype
 * (dequantize_tensor, symmetric.py:272-293).  packed != 0: INT4 storage.
 */
int llq_dequantize(const int8_t* q, const float* scale, int64_t rows, int64_t K, int bits,
                   int group_size, int packed, void* out, int out_dtype, void* stream);

/* pack_int4 / unpack_int4 (symmetric.py:296-346); n = number of int4 values. */
int llq_pack_int4(const int8_t* values, int64_t n, int8_t* packed, int32_t* range_error,
                  void* stream);
int llq_unpack_int4(const int8_t* packed, int64_t n, int8_t* values, void* stream);

/* ------------------------------------------------------------------------ */
/* Routing.                                                                  */
/* ------------------------------------------------------------------------ */

/*
 * Router of the external TritonFusedMoEBlock as RouterCapture recomputes it
 * (src/LLaDA_Quant/trajectory/llada.py:225-234): logits = gate(x) in bf16
 * (fp32 accumulation, one rounding), p = softmax(logits + bias) in fp32,
 * top-k (larger value first, ties to the smaller expert id).  x bf16 [T, H],
 * gate_w bf16 [E, H], bias float32 [E] or NULL, logits bf16 [T, E] or NULL.
 * renormalize != 0 divides the k weights by their sum.  E <= 256, k <= E.
 */
int llq_route(const void* x, const void* gate_w, int64_t T, int H, int E, int k,
              const float* bias, int renormalize, void* logits, float* topk_w,
              int32_t* topk_ids, void* stream);

/* Softmax + top-k from given logits (bf16 or f32) [T, E]. */
int llq_route_topk(const void* logits, int logits_dtype, int64_t T, int E, int k,
                   const float* bias, int renormalize, float* topk_w, int32_t* topk_ids,
                   void* stream);

/*
 * moe_align_block_size of the external fused_moe (described in
 * INFERENCE_REPO_CHANGES.md:274-278): group the T*k (token, slot) entries by
 * expert, stable in entry order.  expert_offsets int32 [E+1]; sorted_slots
 * int32 [T*k] holds token*k + slot.  workspace >= llq_align_workspace_size.
 */
size_t llq_align_workspace_size(int64_t T, int k, int E);
int llq_moe_align(const int32_t* topk_ids, int64_t T, int k, int E, int32_t* expert_offsets,
                  int32_t* sorted_slots, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Permute: x_sorted[p] = x[sorted_slots[p] / k], bf16 rows of H.  kperm != 0
 * also reorders each 8-element block as [0,4,1,5,2,6,3,7], the K order that the
 * LLQ_GEMM_TCGEN05_FAST GEMMs expect (GEMM1 in that mode writes h already so).
 */
int llq_moe_permute(const void* x, int64_t T, int H, int k, const int32_t* sorted_slots,
                    int kperm, void* x_sorted, void* stream);

/* Unpermute/combine: out[t] = bf16(sum_j y_slots[t*k + j]) in fp32, slot order. */
int llq_moe_combine(const void* y_slots, int64_t T, int k, int H, void* out, void* stream);

/*
 * Expert parallelism (new work; the reference has no distributed MoE path --
 * its external serving code only mentions rank-local experts,
 * README.md:496-498).  llq_ep_pack: given sorted_slots from llq_moe_align over
 * destination ranks (topk_ids / experts_per_rank), write each (token, slot)
 * entry's row in that order, its expert id local to the destination rank, its
 * routed weight, and inv_pos[token*k + slot] = its position.  llq_ep_combine:
 * out[t] = bf16(sum_j back_rows[inv_pos[t*k + j]]) in fp32, slot order.
 */
int llq_ep_pack(const void* x, const int32_t* topk_ids, const float* topk_w, int64_t T, int k,
                int H, int experts_per_rank, const int32_t* sorted_slots, void* send_rows,
                int32_t* local_ids, float* weights, int32_t* inv_pos, void* stream);
int llq_ep_combine(const void* back_rows, const int32_t* inv_pos, int64_t T, int k, int H,
                   void* out, void* stream);

/*
 * Expert parallelism over NVLink peer memory (new work, like llq_ep_pack; it
 * is the "ep_dispatch / ep_combine" pair of the custom-op surface, without a
 * collective library or a host synchronisation on the data path).
 *
 * Each rank allocates one exchange window of llq_ep_window_bytes(world, cap, H)
 * with llq_ipc_alloc, passes the llq_ipc_handle_bytes()-byte handle to its
 * peers (any host channel), maps theirs with llq_ipc_open, and keeps a device
 * array `peers[world]` of the window bases (its own at [rank]).  cap = the
 * most (token, slot) entries one rank sends per call (T*k).  One layer call,
 * with an epoch that starts at 1 and grows by one per call on every rank:
 *   llq_ep_dispatch      rows + (local expert id, weight) -> the owners' windows
 *   llq_ep_experts       wait for every rank's dispatch; local experts; GEMM2
 *                        stores each result into its source rank's window
 *   llq_ep_combine_wait  wait for every rank's results; out[t] = sum over slots
 * Waits are bounded (llq_ep_set_timeout_ms, 5 s by default); when one runs out
 * the kernel records a code in the device error word and carries on.  A
 * window serves one stream at a time.  rows_hint: the rows expected on this
 * rank (T*k for balanced routing; picks the token-tile width).
 */
size_t llq_ep_window_bytes(int world, int cap, int H);
int llq_ep_set_timeout_ms(int ms);
int llq_ipc_handle_bytes(void);
int llq_ipc_alloc(size_t bytes, void** ptr, void* handle);
int llq_ipc_open(const void* handle, void** ptr);
int llq_ipc_close(void* ptr);
int llq_ipc_free(void* ptr);
int llq_ep_dispatch(const void* x, const int32_t* topk_ids, const float* topk_w, int64_t T, int k,
                    int H, int experts_per_rank, void* window, void* const* peers, int rank,
                    int world, int cap, uint32_t epoch, int32_t* inv_pos, void* stream);
size_t llq_ep_experts_workspace_size(int world, int cap, int E_local, int H, int I);
int llq_ep_experts(void* window, void* const* peers, int rank, int world, int cap, uint32_t epoch,
                   const int8_t* qw1, const float* sw1, const int8_t* qw2, const float* sw2,
                   int E_local, int H, int I, int bits, int group_size, int64_t rows_hint,
                   void* workspace, size_t workspace_bytes, int impl, void* stream);
int llq_ep_combine_wait(void* window, int rank, int world, int cap, uint32_t epoch,
                        const int32_t* inv_pos, int64_t T, int k, int H, void* out, void* stream);

/* ------------------------------------------------------------------------ */
/* Grouped W4A16 / W8A16 expert GEMMs over the packed buffers.                */
/* ------------------------------------------------------------------------ */

/*
 * GEMM1 of the external fused_moe with the SiLU epilogue
 * (INFERENCE_REPO_CHANGES.md:37-59, 296-309) reading PACKED w1 directly
 * (replaces runtime/moe.py:199-216 + the bf16 fused_moe_kernel):
 * for every sorted row p of expert e,
 *   gate = bf16(x_sorted[p] . W1[e, n]),  up = bf16(x_sorted[p] . W1[e, I+n]),
 *   h_sorted[p, n] = bf16(bf16(silu(gate)) * up)
 * with W1 = bf16(q * scale) exactly as dequantize_tensor.
 * qw1 int8 [E, 2I, H/2 or H], sw1 float32 [E, 2I, H/group].
 * With impl LLQ_GEMM_TCGEN05_FAST, x_sorted must come from llq_moe_permute
 * with kperm != 0, and h_sorted is written in that K order for GEMM2.
 */
int llq_moe_gemm1(const void* x_sorted, const int32_t* expert_offsets, int64_t n_rows, int E,
                  int H, int I, const int8_t* qw1, const float* sw1, int bits, int group_size,
                  void* h_sorted, int impl, void* stream);

/*
 * GEMM2 with MUL_ROUTED_WEIGHT (INFERENCE_REPO_CHANGES.md:259-265), scattered
 * back to (token, slot) order: y_slots[sorted_slots[p]] =
 * bf16((h_sorted[p] . W2[e]) * topk_w[sorted_slots[p]]).
 * qw2 int8 [E, H, I/2 or I], sw2 float32 [E, H, I/group].
 */
int llq_moe_gemm2(const void* h_sorted, const int32_t* expert_offsets,
                  const int32_t* sorted_slots, const float* topk_w, int64_t n_rows, int E,
                  int H, int I, const int8_t* qw2, const float* sw2, int bits, int group_size,
                  void* y_slots, int impl, void* stream);

/*
 * Dense QuantLinear forward on the same kernel (replaces runtime/linear.py:127-131,
 * F.linear(x, dequantize_weight()) without the bias add): out[m, n] =
 * bf16(sum_k x[m, k] * bf16(q[n, k] * s[n, k / group])), fp32 accumulation.
 * x bf16 [M, K], qweight int8 [N, K/2 or K], scale fp32 [N, K/group], out bf16 [M, N].
 * Exact weights only (LLQ_GEMM_AUTO or LLQ_GEMM_TCGEN05); K % 128 == 0, K <= 2048,
 * N % 256 == 0, group % 128 == 0 (others return LLQ_EUNSUPPORTED).  When the layer
 * has fewer output tiles than SMs, K is split into slices whose fp32 partial sums
 * go to the workspace (llq_quant_linear_workspace_size bytes, 0 when unsplit) and
 * are added in slice order by a second kernel.
 */
size_t llq_quant_linear_workspace_size(int64_t M, int K, int N);
int llq_quant_linear(const void* x, int64_t M, int K, int N, const int8_t* qweight,
                     const float* scale, int bits, int group_size, void* out, void* workspace,
                     size_t workspace_bytes, int impl, void* stream);

/*
 * GEMM1 and GEMM2 above in one persistent launch (exact weights): the GEMM2 work
 * of a token tile starts as soon as that tile's h rows are stored, so the two
 * GEMMs share the SMs instead of meeting at a launch boundary.  Same arguments as
 * the pair, plus `counters`: int32 [llq_moe_gemm12_counters(n_rows, E)] of device
 * memory, zero-filled before the first call (every call leaves it zeroed).
 */
size_t llq_moe_gemm12_counters(int64_t n_rows, int E);
int llq_moe_gemm12(const void* x_sorted, const int32_t* expert_offsets,
                   const int32_t* sorted_slots, const float* topk_w, int64_t n_rows, int E,
                   int H, int I, const int8_t* qw1, const float* sw1, const int8_t* qw2,
                   const float* sw2, int bits, int group_size, void* h_sorted, void* y_slots,
                   int32_t* counters, void* stream);

/* ------------------------------------------------------------------------ */
/* Whole layer.                                                              */
/* ------------------------------------------------------------------------ */

/* Workspace bytes for llq_fused_moe_packed. */
size_t llq_moe_workspace_size(int64_t T, int k, int E, int H, int I);

/*
 * fused_moe(hidden_states, w1, w2, gating_output, topk_ids) on PACKED weights
 * (signature: INFERENCE_REPO_CHANGES.md:109-111; PACKED property:
 * runtime/moe.py:199-216): align -> permute -> GEMM1 -> GEMM2 -> combine.
 * x bf16 [T, H], topk_w float32 [T, k], topk_ids int32 [T, k], out bf16 [T, H].
 */
int llq_fused_moe_packed(const void* x, const int8_t* qw1, const float* sw1, const int8_t* qw2,
                         const float* sw2, const float* topk_w, const int32_t* topk_ids,
                         int64_t T, int E, int H, int I, int k, int bits, int group_size,
                         void* out, void* workspace, size_t workspace_bytes, int impl,
                         void* stream);

/*
 * The PACKED MoE block's forward, router included: logits = x . gate_w^T,
 * softmax(+ bias), top-k, then the routed experts as llq_fused_moe_packed.
 * It replaces the block forward that runs the router
 * (trajectory/llada.py:225-234 restates it) and then calls fused_moe
 * (INFERENCE_REPO_CHANGES.md:109-111), in one call: router, alignment,
 * permute, expert GEMMs and combine on one stream.  gate_w bf16 [E, H];
 * bias float32 [E] or NULL; logits bf16 [T, E] or NULL (written when given);
 * topk_w float32 [T, k] and topk_ids int32 [T, k] are written (the routing the
 * experts consumed); workspace as for llq_fused_moe_packed (same size).
 */
int llq_moe_block_packed(const void* x, const void* gate_w, const float* bias, int renormalize,
                         int64_t T, int E, int H, int I, int k, const int8_t* qw1,
                         const float* sw1, const int8_t* qw2, const float* sw2, int bits,
                         int group_size, void* logits, float* topk_w, int32_t* topk_ids,
                         void* out, void* workspace, size_t workspace_bytes, int impl,
                         void* stream);

/*
 * No counterpart in the reference.  The same layer as llq_fused_moe_packed for
 * callers that cannot allocate device memory (a plugin inside a framework that
 * owns the allocator, a runtime that reserves all memory at start-up): no
 * workspace argument, and the library allocates nothing either.  Its scratch is
 * one fixed device array of about 12 MiB inside the library, held on every GPU
 * that loads it until exit.  Limits: T*k <= 2048, H <= 2048, I <= 1024,
 * E <= 256; larger calls return LLQ_EINVAL.  The first call on a device sets
 * up the array's address there -- make it before any stream capture.  All
 * calls share the array: calls whose GPU executions overlap race.
 */
int llq_fused_moe_packed_noalloc(const void* x, const int8_t* qw1, const float* sw1,
                                 const int8_t* qw2, const float* sw2, const float* topk_w,
                                 const int32_t* topk_ids, int64_t T, int E, int H, int I, int k,
                                 int bits, int group_size, void* out, int impl, void* stream);

/*
 * Device error word written by bounded waits inside the tcgen05 kernels
 * (0 = none).  Reading it synchronizes the device.  llq_clear_device_error
 * resets it.
 */
int llq_device_error(int32_t* code);
int llq_clear_device_error(void);

#ifdef __cplusplus
}
#endif

#endif /* LLADA_QUANT_H */
