/*
 * aiter_b200 -- C ABI of the B200 (sm_100a) fused-MoE hot path.
 *
 * Every entry point mirrors a ctypes-mode operator of the reference
 * (aiter/jit/core.py:1105-1363): tensors are passed as `aiter_tensor_t*`
 * (NULL for None), Python ints as int64_t (-1 for None), bools as int,
 * floats as float, strings as const char* (may be NULL), and the CUDA stream is
 * appended last.  Each call returns 0 on success and -1 on error; the message is
 * kept in thread-local storage and read with aiter_get_last_error()
 * (csrc/include/aiter_ctypes_error.h:56-130).  Exceptions never cross this
 * boundary.  Kernels never allocate or free caller memory; every output tensor is
 * owned by the caller.
 */
#ifndef AITER_B200_H
#define AITER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types: same values as AiterDtype (csrc/include/aiter_enum.h:26-41). */
typedef enum {
    AITER_DTYPE_fp8 = 0,      /* float8_e4m3fn */
    AITER_DTYPE_fp8_e8m0 = 1,
    AITER_DTYPE_fp16 = 2,
    AITER_DTYPE_bf16 = 3,
    AITER_DTYPE_fp32 = 4,
    AITER_DTYPE_i4x2 = 5,
    AITER_DTYPE_fp4x2 = 6,    /* two e2m1 values per byte, element 2i in the low nibble */
    AITER_DTYPE_u32 = 7,
    AITER_DTYPE_i32 = 8,
    AITER_DTYPE_i16 = 9,
    AITER_DTYPE_i8 = 10,
    AITER_DTYPE_u8 = 11,
    AITER_DTYPE_i64 = 12,
    AITER_DTYPE_u64 = 13
} AiterDtype;

/* Activation / quantisation enums (csrc/include/aiter_enum.h:7-25). */
enum { AITER_ACT_NO = -1, AITER_ACT_SILU = 0, AITER_ACT_GELU = 1, AITER_ACT_SWIGLU = 2 };
enum {
    AITER_QUANT_NO = 0, AITER_QUANT_PER_TENSOR = 1, AITER_QUANT_PER_TOKEN = 2,
    AITER_QUANT_PER_1X32 = 3, AITER_QUANT_PER_1X128 = 4, AITER_QUANT_PER_128X128 = 5
};

/* Tensor descriptor, byte-compatible with aiter_tensor_t
 * (csrc/include/aiter_tensor.h:8-18; 160 bytes, aiter/utility/aiter_types.py:68-86).
 * Strides are in elements; `ptr` is device memory. */
typedef struct aiter_tensor_t {
    void* ptr;
    size_t numel_;
    int ndim;
    int64_t shape[8];
    int64_t strides[8];
    int dtype_;
    int device_id;
} aiter_tensor_t;

/* ---- error bridge: csrc/include/aiter_ctypes_error.h:56-67 ---------------- */
int aiter_ctypes_abi_version(void);            /* returns 2 */
const char* aiter_get_last_error(void);        /* NULL when no error */
void aiter_clear_last_error(void);

/* Device-side error word of the bounded waits inside the kernels: 0 = none,
 * 1 = a wait ran out of time (the kernel then returned early).  `clear` resets it.
 * Has no counterpart in the reference, whose waits are unbounded
 * (csrc/include/custom_all_reduce.cuh:150-252). */
int aiter_device_error(int clear);

/* ---- routing ------------------------------------------------------------- */

/* Replaces aiter.topk_softmax (aiter/ops/moe_op.py:15-24 ->
 * csrc/kernels/topk_softmax_kernels.cu:760).  gating_output [M, E(+shared)]
 * bf16/fp16/fp32 (row stride allowed); topk_weights [M, k(+shared)] f32,
 * topk_indices [M, k] i32, token_expert_indices [M, k] i32 (= slot*M + row).
 * Ties resolve to the lower expert index. */
int topk_softmax(aiter_tensor_t* topk_weights, aiter_tensor_t* topk_indices,
                 aiter_tensor_t* token_expert_indices, aiter_tensor_t* gating_output,
                 int need_renorm, int64_t num_shared_experts,
                 const char* shared_expert_scoring_func, void* stream);

/* Replaces aiter.grouped_topk (aiter/ops/topk.py:28-38 ->
 * csrc/kernels/topk_softmax_kernels_group.cu:1265-1300). */
int grouped_topk(aiter_tensor_t* gating_output, aiter_tensor_t* topk_weights,
                 aiter_tensor_t* topk_ids, int64_t num_expert_group, int64_t topk_group,
                 int need_renorm, int is_softmax, float routed_scaling_factor, void* stream);

/* Replaces aiter.biased_grouped_topk (aiter/ops/topk.py:15-25 / :75-113 ->
 * csrc/kernels/topk_softmax_kernels_group.cu:1219-1263). */
int biased_grouped_topk(aiter_tensor_t* gating_output, aiter_tensor_t* correction_bias,
                        aiter_tensor_t* topk_weights, aiter_tensor_t* topk_ids,
                        int64_t num_expert_group, int64_t topk_grp, int need_renorm,
                        float routed_scaling_factor, void* stream);

/* Replaces aiter.topk_sigmoid (aiter/ops/moe_op.py:40-42 ->
 * csrc/py_itfs_ck/topk_sigmoid_kernels.cu:15-66): per token the topk largest logits of
 * gating_output [tokens, experts <= 1024] (fp32/bf16/fp16, contiguous), in descending
 * order (equal values: lower expert first), topk_indices [tokens, topk] i32 and
 * topk_weights [tokens, topk] (fp32/bf16/fp16) = sigmoid(logit) computed in fp32. */
int topk_sigmoid(aiter_tensor_t* topk_weights, aiter_tensor_t* topk_indices, aiter_tensor_t* gating_output,
                 void* stream);

/* Replaces aiter.moe_sum (aiter/ops/moe_op.py:45-46 -> csrc/kernels/topk_softmax_kernels.cu:
 * 737-854): output [tokens, hidden] = sum over the topk slots of input [tokens, topk,
 * hidden] (fp32/bf16/fp16); for topk 2, 4 and 5 the sum is rounded to the element type
 * after every slot, as the reference's kernel adds in the element type; otherwise it
 * accumulates in fp32 and rounds once, as its at::sum_out fallback. */
int moe_sum(aiter_tensor_t* input, aiter_tensor_t* output, void* stream);

/* ---- sorting ------------------------------------------------------------- */

/* Workspace bytes moe_sorting_fwd needs for these sizes (0 = none).
 * Replaces moe_sorting_get_workspace_size (csrc/py_itfs_ck/moe_sorting_kernels.cu:35). */
int64_t moe_sorting_get_workspace_size(int64_t num_tokens, int64_t num_experts, int64_t topk,
                                       int64_t dispatch_policy);

/* Replaces aiter.moe_sorting_fwd (aiter/ops/moe_sorting.py:11-24 ->
 * csrc/py_itfs_ck/moe_sorting_kernels.cu:10-76).  Outputs are written in place;
 * moe_buf[:tokens] is zeroed.  `workspace` (u8/i32, >= the size above) is the
 * scratch the reference binding allocates itself; it may be NULL when the size
 * above is 0.  num_local_tokens is read on the device (no host sync).
 * token_sorted_pos (optional, i32 [M*topk]; no reference counterpart) receives the
 * sorted row of every (token, slot), -1 when the slot's expert is masked out: the
 * map moe_gather_quant_1x128 uses to write each token's row once per slot. */
int moe_sorting_fwd(aiter_tensor_t* topk_ids, aiter_tensor_t* topk_weights,
                    aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_weights,
                    aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                    aiter_tensor_t* moe_buf, int64_t num_experts, int64_t unit_size,
                    aiter_tensor_t* local_expert_mask, aiter_tensor_t* num_local_tokens,
                    int64_t dispatch_policy, aiter_tensor_t* workspace,
                    aiter_tensor_t* token_sorted_pos, void* stream);

/* moe_sorting_fwd without a workspace argument, for callers that cannot allocate
 * device memory while they run (a serving engine that gave all free HBM to its
 * KV-cache pool at start-up, a C host without its own device allocator).  It has
 * no counterpart in the reference, whose binding allocates the workspace with
 * torch.  The histograms use a 1 MiB array inside the library; inputs needing more
 * (moe_sorting_get_workspace_size > 1 MiB, i.e. ceil(M / floor(1024 / topk)) * E >
 * 262144 when the multi-CTA sort runs) are rejected with an error.  CUDA loads the
 * library's code lazily, so the array is placed on a GPU by the first call of this
 * function on that device (any input size, e.g. one token): make that call at
 * start-up, before the free HBM is taken and before any stream capture.  The
 * array's address is cached per device (ids 0..63) and looked up again under a
 * new CUDA context.  All calls share the array, so calls that overlap on the GPU
 * race.  No cudaMalloc/cudaFree or other allocation is made. */
int moe_sorting_fwd_static_scratch(aiter_tensor_t* topk_ids, aiter_tensor_t* topk_weights,
                                   aiter_tensor_t* sorted_token_ids, aiter_tensor_t* sorted_weights,
                                   aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                                   aiter_tensor_t* moe_buf, int64_t num_experts, int64_t unit_size,
                                   aiter_tensor_t* local_expert_mask, aiter_tensor_t* num_local_tokens,
                                   int64_t dispatch_policy, aiter_tensor_t* token_sorted_pos,
                                   void* stream);

/* ---- quantisation -------------------------------------------------------- */

/* Replaces aiter.dynamic_per_token_scaled_quant as per_group_quant_hip drives it
 * (aiter/ops/quant.py:261-292,473-481 -> csrc/kernels/quant_kernels.cu:20-133):
 * input viewed as [rows, group] bf16/fp16/fp32 -> out fp8 e4m3fn, scales f32
 * [rows] (= [M, K/group]); scale = amax/448 (0 -> 1), q = x / scale.
 * shuffle_scale writes scales transposed ([K/group, M]).  num_rows (device i32
 * [1], may be NULL) limits the rows processed to num_rows[0]*num_rows_factor*K/group. */
int dynamic_per_token_scaled_quant(aiter_tensor_t* out, aiter_tensor_t* input,
                                   aiter_tensor_t* scales, aiter_tensor_t* scale_ub,
                                   int shuffle_scale, aiter_tensor_t* num_rows,
                                   int64_t num_rows_factor, void* stream);

/* 1x128 fp8 quantisation of the activations, scattered into sorted-row order: the
 * A operand of stage 1.  Replaces the activation quant of fused_moe_2stages
 * (aiter/fused_moe.py:1201-1209 -> per_group_quant_hip, aiter/ops/quant.py:261-292)
 * together with the row gather the CK stage-1 kernel does internally
 * (gemm_moe_ck2stages_common_blockscale.cuh:9-180).  Each token is quantised once
 * and stored to the sorted rows token_sorted_pos[token*topk + slot] (from
 * moe_sorting_fwd; -1 = skip).
 * hidden [M, D] bf16/fp16/fp32, or fp8 with hidden_scale [M, D/128] f32 (copied);
 * out [rows, D] fp8 and out_scale [D/128, rows] f32; padding rows are not written
 * (the GEMMs never store their results). */
int moe_gather_quant_1x128(aiter_tensor_t* hidden, aiter_tensor_t* hidden_scale,
                           aiter_tensor_t* token_sorted_pos, int64_t topk,
                           aiter_tensor_t* out, aiter_tensor_t* out_scale, void* stream);

/* MXFP4 activation quant: per 32-element group e = e8m0(amax / 4) (the reference's
 * round-half-up rule), codes e2m1(x / 2^(e-127)) round-to-nearest-even saturating at
 * 6, packed two per byte low nibble first; scales in row order [rows, cols/32] or, with
 * shuffle_scale, in the e8m0_shuffle layout of a [rows padded to 32, cols/32 padded
 * to 8] matrix.  Rows from num_rows[0] * num_rows_factor on are skipped.  group_size
 * must be 32.  Replaces dynamic_per_group_scaled_quant_fp4 (aiter/ops/quant.py:485-497;
 * semantics of per_1x32_f4_quant, :75-106). */
int dynamic_per_group_scaled_quant_fp4(aiter_tensor_t* out, aiter_tensor_t* input, aiter_tensor_t* scales,
                                       int64_t group_size, int shuffle_scale, aiter_tensor_t* num_rows,
                                       int64_t num_rows_factor, void* stream);
/* e8m0 scales [token_num or token_num * topk, cols/32] gathered into moe_sorting order
 * and shuffled: out_scale [ceil(len(sorted_ids)/32)*32, cols/32]; padding slots and
 * rows from num_valid_ids[0] on are 0.  Replaces mxfp4_moe_sort_hip
 * (aiter/ops/quant.py:552-563; layout of op_tests/test_moe_sorting_mxfp4.py:20-43). */
int mxfp4_moe_sort_hip(aiter_tensor_t* out_scale, aiter_tensor_t* scale, aiter_tensor_t* sorted_ids,
                       aiter_tensor_t* num_valid_ids, int64_t token_num, int64_t cols, void* stream);
/* Both in one launch: out [rows, cols/2] fp4x2 of every input row (rows = token_num,
 * or token_num * topk), scales sorted and shuffled as mxfp4_moe_sort_hip writes them.
 * Replaces fused_dynamic_mxfp4_quant_moe_sort_hip (aiter/ops/quant.py:584-597). */
int fused_dynamic_mxfp4_quant_moe_sort_hip(aiter_tensor_t* out, aiter_tensor_t* scales, aiter_tensor_t* input,
                                           aiter_tensor_t* sorted_ids, aiter_tensor_t* num_valid_ids,
                                           int64_t token_num, int64_t block_m, int64_t group_size, void* stream);

/* A8W4 weight preparation: MXFP4 weights (e2m1 packed two per byte, low nibble
 * first, + e8m0 scale per 32 along K; per_1x32_f4_quant, aiter/ops/quant.py:75-106)
 * -> e4m3 [E, N, K] with a power-of-two f32 scale per 128x128 block, the operand
 * format of the FP8 grouped GEMMs.  Exact for blocks whose non-zero group
 * exponents span <= 14 binades; `status` (optional i32 [1], accumulated) counts
 * blocks that are not.  Runs once per weight, like the reference's shuffle_weight
 * (aiter/ops/shuffle.py:7-27). */
int mxfp4_to_fp8_blockscale(aiter_tensor_t* w_fp4, aiter_tensor_t* w_scale, aiter_tensor_t* out,
                            aiter_tensor_t* out_scale, aiter_tensor_t* status, void* stream);

/* A8W4 scale preparation for the native MXFP4 grouped GEMMs: e8m0 scales [E, N, K/32]
 * -> chunks [E, N/128, K/128, 512] u8, per 128 weight rows x 128 K values the 128 x 4
 * scales as the 32 lines of 16 bytes that tcgen05.cp copies into tensor memory (line
 * r, word w, byte b = scale of row 32w + r, K group b).  The role of the reference's
 * e8m0_shuffle of the weight scales (aiter/utility/fp4_utils.py) for these kernels. */
int mxfp4_moe_weight_scale_chunks(aiter_tensor_t* w_scale, aiter_tensor_t* out, void* stream);

/* ---- grouped GEMMs (FP8 block-scale, tcgen05) ----------------------------- */

/* Stage 1: replaces ck_moe_stage1_fwd + the intermediate requant
 * (aiter/ops/moe_op.py:534-575, aiter/fused_moe.py:1306-1314; CK template
 * csrc/ck_gemm_moe_2stages_codegen/gemm_moe_ck2stages_common_blockscale.cuh:9-180).
 * a1 [rows, D] fp8 + a1_scale [D/128, rows] f32 (from moe_gather_quant_1x128);
 * w1 [E, 2I, D] fp8 + w1_scale [E, 2I/128, D/128] f32; sorted ids / expert ids /
 * num_valid_ids from moe_sorting_fwd with unit_size == block_m (128).
 * Writes, for every real sorted row r, out[r, :] = fp8(act(gate) * up / s) and
 * out_scale[:, r] = s per 128 columns (1x128 requant, s = amax/448); padding rows
 * are not written.  num_tokens = M (the padding id).  activation: AITER_ACT_SILU,
 * AITER_ACT_GELU or AITER_ACT_SWIGLU (aiter/fused_moe.py:1473-1480).  The
 * intermediate is rounded to bf16 before the requant. */
int moe_stage1_fp8_blockscale(aiter_tensor_t* a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1,
                              aiter_tensor_t* w1_scale, aiter_tensor_t* sorted_token_ids,
                              aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                              aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens,
                              int64_t block_m, int64_t activation, void* stream);
/* Stage 1 with the fused_moe options of the reference's stage-1 path
 * (torch_moe_stage1, aiter/fused_moe.py:1483-1585): sorted_weights non-NULL =
 * doweight_stage1 (gate and up of row r multiplied by sorted_weights[r] before the
 * activation; pass NULL weights to stage 2 then); inter_dtype = AITER_DTYPE_bf16 or
 * AITER_DTYPE_fp16, the dtype the intermediate is rounded to before its fp8 requant
 * (the activation dtype of the call). */
int moe_stage1_fp8_blockscale_ex(aiter_tensor_t* a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1,
                                 aiter_tensor_t* w1_scale, aiter_tensor_t* sorted_token_ids,
                                 aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                                 aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens,
                                 int64_t block_m, int64_t activation, aiter_tensor_t* sorted_weights,
                                 int64_t inter_dtype, void* stream);

/* Stage 2: replaces ck_moe_stage2_fwd (aiter/ops/moe_op.py:578-615; CK template
 * gemm_moe_ck2stages_common_blockscale.cuh:330-470).
 * a2 [rows, I] fp8 + a2_scale [I/128, rows] f32 (stage-1 output, sorted rows);
 * w2 [E, D, I] fp8 + w2_scale [E, D/128, I/128] f32.  Adds
 * sorted_weights[r] * (a2[r] @ w2[e]^T) of every real sorted row r into
 * out[token(r)] (bf16 or fp16 [M, D], zeroed by moe_sorting_fwd): the top-k weighted
 * scatter-reduce back to token order.  sorted_weights NULL: weight 1 (after
 * doweight_stage1). */
int moe_stage2_fp8_blockscale(aiter_tensor_t* a2, aiter_tensor_t* a2_scale, aiter_tensor_t* w2,
                              aiter_tensor_t* w2_scale, aiter_tensor_t* sorted_token_ids,
                              aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                              aiter_tensor_t* sorted_weights, aiter_tensor_t* out, int64_t block_m,
                              void* stream);

/* The two stages with the experts' biases (the exp_bias of moe_cktile2stages_gemm1 /
 * gemm2, aiter/ops/moe_op.py:344-465, which fused_moe passes for per_1x32 Swiglu,
 * aiter/fused_moe.py:1228-1238): stage 1 adds bias [E, 2 * inter_dim] f32 to the
 * gate/up GEMM output after the doweight multiply and before the activation; stage 2
 * adds bias [E, model_dim] f32 to the down GEMM output before the top-k weight
 * (torch_moe_stage1/2, aiter/fused_moe.py:1572-1573, 1662-1663). */
int moe_stage1_fp8_blockscale_bias(aiter_tensor_t* a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1,
                                   aiter_tensor_t* w1_scale, aiter_tensor_t* sorted_token_ids,
                                   aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                                   aiter_tensor_t* out, aiter_tensor_t* out_scale, int64_t num_tokens,
                                   int64_t block_m, int64_t activation, aiter_tensor_t* sorted_weights,
                                   int64_t inter_dtype, aiter_tensor_t* bias, void* stream);
int moe_stage2_fp8_blockscale_bias(aiter_tensor_t* a2, aiter_tensor_t* a2_scale, aiter_tensor_t* w2,
                                   aiter_tensor_t* w2_scale, aiter_tensor_t* sorted_token_ids,
                                   aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                                   aiter_tensor_t* sorted_weights, aiter_tensor_t* out, int64_t block_m,
                                   aiter_tensor_t* bias, void* stream);

/* A8W4 stages: replace moe_cktile2stages_gemm1 / gemm2 for MXFP4 weights
 * (aiter/ops/moe_op.py:343-465, called by fused_moe for per_1x32,
 * aiter/fused_moe.py:985-1008).  Same operands and options as the _bias entries
 * except the weights: w1 [E, 2 * inter_dim, D/2] / w2 [E, D, inter_dim/2] fp4x2 (e2m1
 * pairs, low nibble first), read at 4 bits by the TMA, with their scales as chunks
 * from mxfp4_moe_weight_scale_chunks; the scales are applied by
 * tcgen05.mma.kind::mxf8f6f4.block_scale, the activations' 1x128 f32 scales promoted
 * per 128-wide K block.  bias may be NULL. */
int moe_stage1_a8w4(aiter_tensor_t* a1, aiter_tensor_t* a1_scale, aiter_tensor_t* w1,
                    aiter_tensor_t* w1_scale_chunks, aiter_tensor_t* sorted_token_ids,
                    aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids, aiter_tensor_t* out,
                    aiter_tensor_t* out_scale, int64_t num_tokens, int64_t block_m, int64_t activation,
                    aiter_tensor_t* sorted_weights, int64_t inter_dtype, aiter_tensor_t* bias, void* stream);
int moe_stage2_a8w4(aiter_tensor_t* a2, aiter_tensor_t* a2_scale, aiter_tensor_t* w2,
                    aiter_tensor_t* w2_scale_chunks, aiter_tensor_t* sorted_token_ids,
                    aiter_tensor_t* sorted_expert_ids, aiter_tensor_t* num_valid_ids,
                    aiter_tensor_t* sorted_weights, aiter_tensor_t* out, int64_t block_m, aiter_tensor_t* bias,
                    void* stream);

/* ---- gated activations (the split-K tail of the reference's fused_moe) ----- */
/* Replace aiter.silu_and_mul / gelu_and_mul / gelu_tanh_and_mul / scaled_silu_and_mul
 * (aiter/ops/activation.py:10-23 -> csrc/kernels/activation_kernels.cu:24-160, 337-360;
 * used by aiter/fused_moe.py:1719-1724): input [..., 2d] = [x | y] -> out [..., d] =
 * act(x) * y computed in fp32.  fp32 input: out fp32, bf16 or fp16; bf16 / fp16 input:
 * out of the same type.  The scaled form multiplies by 1 / scale[0] (f32 tensor, read on
 * the device) and writes fp8 e4m3 (round to nearest, saturating). */
int silu_and_mul(aiter_tensor_t* out, aiter_tensor_t* input, void* stream);
int gelu_and_mul(aiter_tensor_t* out, aiter_tensor_t* input, void* stream);
int gelu_tanh_and_mul(aiter_tensor_t* out, aiter_tensor_t* input, void* stream);
int scaled_silu_and_mul(aiter_tensor_t* out, aiter_tensor_t* input, aiter_tensor_t* scale, void* stream);

/* ---- bf16 GEMM (the GEMM half of GEMM + allreduce) ------------------------ */
/* out[M, N] = A[M, K] @ W[N, K]^T, bf16 in / fp32 accumulate / bf16 out, on
 * tcgen05 kind::f16.  Replaces tgemm.mm / gemm_a16w16 (aiter/tuned_gemm.py:224-308,
 * 506-529; weights in the F.linear [N, K] layout).  Needs K % 64 == 0 and
 * N % 256 == 0; out may be strided by rows (e.g. an allreduce staging buffer). */
int gemm_a16w16(aiter_tensor_t* a, aiter_tensor_t* w, aiter_tensor_t* out, void* stream);

/* ---- tensor-parallel allreduce over CUDA IPC ------------------------------ */
/* Replaces the reference's HIP-IPC custom allreduce (aiter/ops/custom_all_reduce.py:
 * init_custom_ar / all_reduce / dispose -> csrc/kernels/custom_all_reduce.cu:74-117,
 * csrc/include/custom_all_reduce.cuh:2243-2420).  One process per GPU.
 * custom_ar_init allocates this rank's IPC region (signals + 3 staging buffers of
 * max_bytes: eager calls alternate the first two, calls captured into a CUDA graph
 * use the third and end with a barrier) and writes its 64-byte cudaIpcMemHandle to handle_out; the caller
 * exchanges the handles (the reference uses its CPU group / TCP store,
 * custom_all_reduce.py:140-153,219-240) and passes all `world` of them, in rank
 * order, to custom_ar_open_peers. */
int custom_ar_init(int64_t rank, int64_t world, int64_t max_bytes, int64_t device, int64_t* ctx_out,
                   void* handle_out);
int custom_ar_open_peers(int64_t ctx, const void* handles);
/* Test hook with no reference counterpart: maps every peer slot to this rank's own
 * region, so barriers wait on flags no peer will ever write (exercises the bounded
 * waits on one GPU). */
int custom_ar_open_loopback(int64_t ctx);
/* Staging buffer the next eager all_reduce will use: a producer that writes its
 * bf16 result there and passes it as `inp` skips the input copy. */
int custom_ar_next_buffer(int64_t ctx, int64_t* ptr_out, int64_t* bytes_out);
/* The same for the next call made eagerly (capturing = 0) or during a CUDA graph
 * capture (capturing != 0). */
int custom_ar_next_buffer_ex(int64_t ctx, int64_t capturing, int64_t* ptr_out, int64_t* bytes_out);
/* out = sum over ranks of inp (bf16, fp16 or fp32, accumulated in fp32 in rank order, identical
 * bits on every rank).  force_two_shot: 1 = two-shot (reduce-scatter + all-gather
 * over peer memory), 0 = one-shot, negative = by size (one-shot always at 2 ranks, up to
 * 2 MiB at 3-4 ranks, up to 1 MiB above). */
int custom_ar_all_reduce(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t force_two_shot,
                         void* stream);
/* all_reduce with open_fp8_quant (csrc/kernels/custom_all_reduce.cu:76-115 and
 * allReduceQuantFp8, csrc/include/custom_all_reduce.cuh:1018-1088): fp16 messages of
 * at least 128 * 2048 elements take a two-shot allreduce whose all-gather moves fp8
 * e4m3 codes with one fp16 scale per group of 128 (or 64, 32, 16, 8) elements; each
 * rank's own segment is exact, the others carry the fp8 rounding.  Every other
 * message takes custom_ar_all_reduce's path. */
int custom_ar_all_reduce_fp8(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, void* stream);
/* GEMM + allreduce, out = allreduce(A @ W^T): the GEMM epilogue writes into the
 * staging buffer the allreduce reads, so the partial product is never copied.
 * No reference counterpart (the reference calls tgemm.mm then
 * tensor_model_parallel_all_reduce, aiter/dist/communication_op.py:30-37). */
int custom_ar_gemm_all_reduce(int64_t ctx, aiter_tensor_t* a, aiter_tensor_t* w, aiter_tensor_t* out,
                              int64_t force_two_shot, void* stream);
/* The same GEMM + allreduce as one kernel: the GEMM epilogue pushes its output tiles
 * over NVLink into the peers' staging buffers while later tiles are multiplied
 * (one-shot: to every rank, which then sums all images; two-shot: to the tile's
 * owner rank, which sums and publishes it for every rank to pull).  Same result
 * bits as custom_ar_gemm_all_reduce, which it falls back to when the pushed images
 * do not fit one staging buffer.  Replaces, with custom_ar_gemm_all_reduce, the
 * reference's tgemm.mm + tensor_model_parallel_all_reduce pair
 * (aiter/tuned_gemm.py:506-529, aiter/dist/communication_op.py:30-37). */
int custom_ar_gemm_all_reduce_fused(int64_t ctx, aiter_tensor_t* a, aiter_tensor_t* w, aiter_tensor_t* out,
                                    int64_t force_two_shot, void* stream);
/* Allreduce fused with the residual add and RMSNorm that follow it: res_out =
 * bf16(allreduce(inp) + res_inp), out = bf16(res * weight * rsqrt(mean(res^2) + eps))
 * row by row over the last dimension (hidden <= 16384).  With scale_out given
 * ([rows] f32) `out` is fp8 e4m3 with one scale per row (amax / 448).  Replaces
 * fused_allreduce_rmsnorm / fused_allreduce_rmsnorm_quant
 * (aiter/ops/custom_all_reduce.py:65-94; csrc/include/custom_all_reduce.cuh:1187-1500). */
int custom_ar_allreduce_rmsnorm(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* res_inp, aiter_tensor_t* res_out,
                                aiter_tensor_t* out, aiter_tensor_t* weight, float eps, aiter_tensor_t* scale_out,
                                void* stream);
/* The same with the one-/two-shot choice (the reference's use_1stage): force_two_shot
 * 1 = two-shot (each row reduced by one owner rank, every rank takes the reduced bf16
 * row from it and adds the residual and normalises locally, as the reference's
 * two-stage kernels do, csrc/include/custom_all_reduce.cuh:1187-1250), 0 = one-shot,
 * negative = by size.  Same bits either way. */
int custom_ar_allreduce_rmsnorm_ex(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* res_inp,
                                   aiter_tensor_t* res_out, aiter_tensor_t* out, aiter_tensor_t* weight,
                                   float eps, aiter_tensor_t* scale_out, int64_t force_two_shot, void* stream);
/* All-gather over peer memory (the reference's custom all-gather,
 * aiter/dist/parallel_state.py:492-501, csrc/include/custom_all_reduce.cuh:678-740):
 * inp of any dtype (a multiple of 16 bytes, <= max_bytes), out = the world inputs in
 * rank order along dim 0 (last_dim == 0) or along the last dim (last_dim != 0; input
 * rows a multiple of 16 bytes). */
int custom_ar_all_gather(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t last_dim, void* stream);
/* Reduce-scatter over peer memory (the reference's custom reduce-scatter,
 * aiter/dist/parallel_state.py:511-538): inp [n] bf16 / fp16 / fp32 (n a multiple of
 * world, each share a multiple of 16 bytes), out [n / world] = this rank's share of
 * the rank-ordered fp32 sum (the same bits as those elements of custom_ar_all_reduce). */
int custom_ar_reduce_scatter(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, void* stream);
int custom_ar_dispose(int64_t ctx);
/* Error word of the allreduce barriers (1 = a peer did not arrive within 2 s). */
int custom_ar_device_error(int clear);

/* ---- quick allreduce: two-shot allreduce with quantised NVLink traffic ----- */
/* Replaces the reference's QuickReduce (aiter/ops/quick_all_reduce.py:13-38 ->
 * csrc/kernels/quick_all_reduce.cu:11-98, csrc/include/quick_all_reduce.cuh:581-991;
 * aiter/dist/device_communicators/quick_all_reduce.py:59-268).  One process per GPU,
 * world sizes 2, 4 and 8.  init_custom_qr (reference :11-26) allocates this rank's
 * IPC region (signals + 2 regions of qr_max_size bytes, rounded up to 32 KB; <= 0
 * takes qr_max_size()) on `device` and writes its 64-byte cudaIpcMemHandle to
 * handle_out (the reference's qr_get_handle, :35-43); qr_open_handles (:44-58)
 * takes every rank's handle in rank order. */
int init_custom_qr(int64_t rank, int64_t world, int64_t qr_max_size, int64_t device, int64_t* ctx_out,
                   void* handle_out);
int qr_open_handles(int64_t ctx, const void* handles);
/* out = sum over ranks of inp (fp16 or bf16, same dtype and size, contiguous, a
 * multiple of 16 bytes, not overlapping).  quant_level 0 = FP, 1 = FP8 (e4m3fn),
 * 2 = INT6, 3 = INT4 (any other value = FP, as the reference's dispatch): every
 * rank's contribution and the owner's sum are quantised in groups of 32 with a
 * scale per group; sums run in the arithmetic type (fp16, or bf16 unless
 * cast_bf2half) in rank order.  Every rank gets identical bits.  (:62-93) */
int qr_all_reduce(int64_t ctx, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t quant_level,
                  int64_t cast_bf2half, void* stream);
int qr_destroy(int64_t ctx);
/* Test hook with no reference counterpart: the quick allreduce of `world` ranks
 * emulated on one GPU in one cooperative launch (the ranks' CTAs wait on one another
 * inside a single launch), with private regions.  inp and out are [world, N]; row r
 * of out receives rank r's result.  Synchronous. */
int qr_all_reduce_emulated(int64_t world, aiter_tensor_t* inp, aiter_tensor_t* out, int64_t quant_level,
                           int64_t cast_bf2half, void* stream);
/* Default registered size, 2 GiB (:95-98). */
int64_t qr_max_size(void);
/* Error word of the quick allreduce's peer waits (1 = a peer did not arrive within 2 s). */
int qr_device_error(int clear);

/* ---- expert-parallel dispatch / combine over NVLink ----------------------- */
/* The token all-to-all around an EP fused MoE, replacing the MoRI
 * EpDispatchCombineOp the reference drives (aiter/dist/device_communicators/
 * all2all.py:21-98, op_tests/multigpu_tests/test_dispatch_combine.py:76-171), intra-node.
 * Rank r owns experts [r * experts_per_rank, (r + 1) * experts_per_rank).
 * ep_init allocates this rank's IPC region for tokens of `hidden` elements of
 * token_dtype (fp8, bf16 or fp16) with scale_dim f32 scales each, up to max_tokens
 * per rank, and outputs of comb_dtype (bf16 or fp16); it writes the 64-byte
 * cudaIpcMemHandle; ep_open_handles takes every rank's handle in rank order. */
int ep_init(int64_t rank, int64_t world, int64_t hidden, int64_t token_dtype, int64_t scale_dim,
            int64_t max_tokens, int64_t experts_per_rank, int64_t topk, int64_t comb_dtype, int64_t device,
            int64_t* ctx_out, void* handle_out);
int ep_open_handles(int64_t ctx, const void* handles);
/* ptrs_out[6] = device pointers of this rank's receive arrays: tokens [rows, hidden],
 * scales [rows, scale_dim] f32, ids [rows, topk] i32, weights [rows, topk] f32, the
 * received count (i32 scalar: num_local_tokens of the EP MoE) and the source tags
 * [rows] i32 (source << 24 | token); rows_out = world * max_tokens. */
int ep_buffers(int64_t ctx, int64_t* ptrs_out, int64_t* rows_out);
/* dispatch: tokens [T, hidden], weights [T, topk] f32, scales [T, scale_dim] f32
 * (NULL when scale_dim is 0), ids [T, topk] i32 (global expert ids; others go
 * nowhere), T <= max_tokens.  Every token goes once to every rank owning one of its
 * experts; rank d receives source 0's tokens, then source 1's, ..., in token order.
 * Calls must alternate with ep_combine. */
int ep_dispatch(int64_t ctx, aiter_tensor_t* tokens, aiter_tensor_t* weights, aiter_tensor_t* scales,
                aiter_tensor_t* ids, void* stream);
/* combine: out [>= world * max_tokens, hidden] (row i = output of received row i)
 * -> y [T, hidden], T = the last dispatch's tokens: y[t] = sum over the ranks t went
 * to, in rank order, accumulated in fp32 and rounded once; 0 for a token that went
 * nowhere. */
int ep_combine(int64_t ctx, aiter_tensor_t* out, aiter_tensor_t* y, void* stream);
/* Test hooks with no reference counterpart: `world` ranks emulated on one GPU (the
 * ranks' CTAs run as rows of one cooperative launch), private regions, synchronous.
 * ep_emu_dispatch takes tokens [world, T, hidden], weights / ids [world, T, topk],
 * scales [world, T, scale_dim]; ep_emu_combine takes out [world, world * max_tokens,
 * hidden] and writes y [world, T, hidden]. */
int ep_emu_init(int64_t world, int64_t hidden, int64_t token_dtype, int64_t scale_dim, int64_t max_tokens,
                int64_t experts_per_rank, int64_t topk, int64_t comb_dtype, int64_t device, int64_t* ctx_out);
int ep_emu_buffers(int64_t ctx, int64_t rank, int64_t* ptrs_out, int64_t* rows_out);
int ep_emu_dispatch(int64_t ctx, aiter_tensor_t* tokens, aiter_tensor_t* weights, aiter_tensor_t* scales,
                    aiter_tensor_t* ids, void* stream);
int ep_emu_combine(int64_t ctx, aiter_tensor_t* out, aiter_tensor_t* y, void* stream);
int ep_destroy(int64_t ctx);
/* Error word of the EP kernels' peer waits (1 = a peer did not arrive within 2 s). */
int ep_device_error(int clear);

#ifdef __cplusplus
}
#endif
#endif /* AITER_B200_H */
