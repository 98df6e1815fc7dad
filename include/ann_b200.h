/*
 * ann_b200.h -- C ABI of the B200-native alpakaNN attention path.
 *
 * Every entry point replaces one call of the reference's header-only host API
 * (namespace alpaka::nn::onHost::nn, files include/alpaka/nn/onHost/...) and
 * keeps its argument meaning: same tensors, same extents, same scalar
 * parameters, same default semantics. Views are passed as plain descriptors
 * (pointer, extents, byte pitches), the in-order alpaka queue becomes a CUDA
 * stream handle, and the alpaka executor argument disappears (it only chose
 * alpaka's thread mapping).
 *
 * Conventions
 *  - All data pointers are device pointers (or pointers the device can read,
 *    such as managed memory) unless a function says otherwise.
 *  - ann_view.pitches are BYTE strides per axis, the convention of alpaka's
 *    getPitches(); the innermost pitch of a dense view is sizeof(element).
 *  - Work is enqueued asynchronously on `stream` (NULL = legacy default
 *    stream). Inputs and outputs must stay alive until the stream reaches the
 *    enqueued work, as in the reference (onHost/nn/rope.hpp:88-95).
 *  - Return value: ANN_OK, or an error code. ANN_EINVAL is raised on the host
 *    before anything is enqueued, for exactly the shape conditions on which
 *    the reference throws std::invalid_argument, plus the conditions under
 *    which the reference would read out of bounds (documented per function).
 *    ann_last_error() returns the message of the calling thread's last error.
 *  - The library never falls back to a CPU implementation. Without a usable
 *    CUDA device every compute entry point returns ANN_ECUDA.
 */
#ifndef ANN_B200_H
#define ANN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ANN_B200_VERSION 100 /* 0.1.0 */

#define ANN_OK 0
#define ANN_EINVAL 1  /* shape / argument error (std::invalid_argument in the reference) */
#define ANN_ECUDA 2   /* CUDA runtime error (launch, memcpy, no device)            */
#define ANN_ENOTSUP 3 /* valid request this build does not implement               */
#define ANN_EDEVICE 4 /* a kernel reported an error through the device error word  */
#define ANN_ENCCL 5   /* NCCL error, or a rank that did not join / finish in time  */
#define ANN_EIO 6     /* file error or digest mismatch (std::runtime_error in the reference) */

#define ANN_MAX_RANK 8

/* alpaka::nn::AttentionKvLayout (nn/attention.hpp:10-14) and
 * alpaka::nn::RopeLayout (nn/rope.hpp:10-14) share these values. */
#define ANN_LAYOUT_BTHD 0
#define ANN_LAYOUT_BHTD 1

/* Device error word bits (ann_take_device_error). */
#define ANN_DEVERR_TOKEN_ID 0x1u     /* embeddingLookup saw an id >= vocabulary rows      */
#define ANN_DEVERR_WAIT_TIMEOUT 0x2u /* a kernel gave up waiting for its own copies (1 s) */

typedef void* ann_stream; /* cudaStream_t */
typedef struct ann_comm_s* ann_comm; /* one rank of the node's NCCL communicator */
#define ANN_COMM_ID_BYTES 128        /* size of the rendezvous id (ncclUniqueId)  */

/* Strided view of a tensor: the B200 counterpart of an alpaka IMdSpan
 * (extents from getExtents(), byte pitches from getPitches(), data()). */
typedef struct ann_view {
    void* data;
    int32_t rank;
    int32_t reserved;
    int64_t extents[ANN_MAX_RANK];
    int64_t pitches[ANN_MAX_RANK];
} ann_view;

/* ---- library ---------------------------------------------------------- */

int ann_version(void);
/* Message of the calling thread's last failed call ("" if none). */
const char* ann_last_error(void);
/* Reads and clears the device error word of the current device; synchronises
 * `stream` first. *bits receives the ANN_DEVERR_* bits that were set. */
int ann_take_device_error(ann_stream stream, uint32_t* bits);
/* Self-test of the failure-detection path the kernels share: one CTA waits on
 * an mbarrier with the kernels' bounded wait. arrive != 0: the barrier is
 * arrived on first and the wait completes; arrive == 0: nothing arrives, the
 * wait gives up after limit_ns (at most 2 s) and ANN_DEVERR_WAIT_TIMEOUT shows
 * up in the next ann_take_device_error; the context stays usable. */
int ann_selftest_wait(ann_stream stream, int32_t arrive, uint64_t limit_ns);

/* ---- embeddingLookup: onHost/nn/embedding.hpp:17-36 --------------------
 * out[t, h] = embedding[ids[t], h]. ids: rank-1 uint32; embedding, output:
 * rank 2. Throws (ANN_EINVAL) unless output = [len(ids), embedding.H]
 * (embedding.hpp:23-27). The reference does not range-check ids; here an id
 * >= embedding rows writes zeros to its output row and sets
 * ANN_DEVERR_TOKEN_ID instead of reading out of bounds. Bit-exact copy. */
int ann_embedding_lookup_f32(ann_stream stream, const ann_view* token_ids, const ann_view* embedding,
                             const ann_view* output);
int ann_embedding_lookup_f64(ann_stream stream, const ann_view* token_ids, const ann_view* embedding,
                             const ann_view* output);

/* ---- embeddingLookup -> rmsNorm, fused -----------------------------------
 * out[t, :] = rmsNorm(embedding[ids[t], :], weight, eps) in one launch: the
 * path's first two calls (embedding.hpp:17-36 then rms_norm.hpp:17-35) without
 * the hidden state's round trip through memory, bit for bit their two-launch
 * result. Throws on the conditions of either call; an id >= embedding rows
 * gives a zero output row and ANN_DEVERR_TOKEN_ID. */
int ann_embedding_rms_norm_f32(ann_stream stream, const ann_view* token_ids, const ann_view* embedding,
                               const ann_view* weight, const ann_view* output, float epsilon);
int ann_embedding_rms_norm_f64(ann_stream stream, const ann_view* token_ids, const ann_view* embedding,
                               const ann_view* weight, const ann_view* output, double epsilon);

/* ---- rmsNorm: onHost/nn/rms_norm.hpp:17-35 ----------------------------
 * y = x * rsqrt(sum(x^2)/H + eps) * w[h] along the last axis of any rank.
 * Throws on in/out extent mismatch or weight not rank-1 [H]. */
int ann_rms_norm_f32(ann_stream stream, const ann_view* input, const ann_view* weight, const ann_view* output,
                     float epsilon);
int ann_rms_norm_f64(ann_stream stream, const ann_view* input, const ann_view* weight, const ann_view* output,
                     double epsilon);

/* ---- rope (out of place): onHost/nn/rope.hpp:49-62 ---------------------
 * Interleaved-pair rotation with caller tables cos/sin[position][D/2],
 * position = position_offset + token index (axis 1 for BTHD, axis 2 for
 * BHTD). Validation follows validateRopeShape (rope.hpp:21-46) with the
 * coverage check taken on the layout's real token axis. */
int ann_rope_f32(ann_stream stream, const ann_view* in, const ann_view* cos_table, const ann_view* sin_table,
                 const ann_view* out, int32_t layout, uint32_t position_offset);
int ann_rope_f64(ann_stream stream, const ann_view* in, const ann_view* cos_table, const ann_view* sin_table,
                 const ann_view* out, int32_t layout, uint32_t position_offset);

/* ---- ropeInPlace: onHost/nn/rope.hpp:96-135 ---------------------------
 * Rotates q and (if k != NULL) k in place, in ONE launch and without the
 * reference's temporary buffer + copy. k may have a different head count. */
int ann_rope_inplace_f32(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* cos_table,
                         const ann_view* sin_table, int32_t layout, uint32_t position_offset);
int ann_rope_inplace_f64(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* cos_table,
                         const ann_view* sin_table, int32_t layout, uint32_t position_offset);

/* ---- attentionScores: onHost/nn/attention.hpp:54-81 --------------------
 * scores[b,hq,i,j] = sum_d Q[b,i,hq,d] * K(b,j,hq/g,d), unscaled. Q BTHD;
 * K BTHD [B,Tk,Hkv,D] or BHTD [B,Hkv,Tk,D]. Throws if g == 0 (as the
 * reference) and, unlike the reference, if Q/K extents do not cover the
 * scores grid (the reference reads out of bounds there). */
int ann_attention_scores_f32(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* scores,
                             uint32_t queries_per_kv_group, int32_t kv_layout);
int ann_attention_scores_f64(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* scores,
                             uint32_t queries_per_kv_group, int32_t kv_layout);

/* ---- ops::scale: onHost/ops/elementwise.hpp:330-334 --------------------
 * out = in * scalar (in == out allowed). Throws on extent mismatch. */
int ann_scale_f32(ann_stream stream, const ann_view* in, float scalar, const ann_view* out);
int ann_scale_f64(ann_stream stream, const ann_view* in, double scalar, const ann_view* out);

/* ---- softmax: onHost/nn/softmax.hpp:26-40 ------------------------------
 * Row softmax along `axis` (max-subtracted, exp, divide by the sum; here one
 * reciprocal of the sum per row, within an ulp of the quotient). Rows that
 * are 16-byte aligned, of up to 200 KB (input + mask), are brought into shared
 * memory by bulk copies with bounded waits (also for causalSoftmax and
 * maskedSoftmax): a copy that has not landed after 1 s sets
 * ANN_DEVERR_WAIT_TIMEOUT (ann_take_device_error). */
int ann_softmax_f32(ann_stream stream, const ann_view* in, const ann_view* out, uint32_t axis);
int ann_softmax_f64(ann_stream stream, const ann_view* in, const ann_view* out, uint32_t axis);

/* ---- causalSoftmax: onHost/nn/softmax.hpp:59-80 ------------------------
 * As softmax, with element i of a row masked (output 0, excluded from max
 * and sum) iff idx[query_axis] < idx[key_axis] for idx with idx[axis] = i
 * (top-left aligned, onAcc/internal/nn/softmax.hpp:23-30). */
int ann_causal_softmax_f32(ann_stream stream, const ann_view* in, const ann_view* out, uint32_t axis,
                           uint32_t query_axis, uint32_t key_axis);
int ann_causal_softmax_f64(ann_stream stream, const ann_view* in, const ann_view* out, uint32_t axis,
                           uint32_t query_axis, uint32_t key_axis);

/* ---- maskedSoftmax: onHost/nn/softmax.hpp:42-57 -------------------------
 * Softmax along `axis` of in + mask (an additive mask with the input's
 * extents, e.g. 0 / -inf): max from lowest() over every element, exp of
 * (in + mask - max), divided by the row sum. ANN_EINVAL "maskedSoftmax shape
 * mismatch." unless in, mask and out share extents. */
int ann_masked_softmax_f32(ann_stream stream, const ann_view* in, const ann_view* mask, const ann_view* out,
                           uint32_t axis);
int ann_masked_softmax_f64(ann_stream stream, const ann_view* in, const ann_view* mask, const ann_view* out,
                           uint32_t axis);

/* ---- attentionApply: onHost/nn/attention.hpp:83-110 -------------------
 * out[b,i,hq,d] = sum_j probs[b,hq,i,j] * V(b,j,hq/g,d) over all Tk keys. */
int ann_attention_apply_f32(ann_stream stream, const ann_view* probs, const ann_view* values, const ann_view* out,
                            uint32_t queries_per_kv_group, int32_t kv_layout);
int ann_attention_apply_f64(ann_stream stream, const ann_view* probs, const ann_view* values, const ann_view* out,
                            uint32_t queries_per_kv_group, int32_t kv_layout);

/* ---- gemm: onHost/matrix/gemm.hpp:28-33 (qkvProjection's building block)
 * C = A * B, row-major rank-2 views with unit column stride. Runs on cuBLAS,
 * loaded at first use; ANN_ENOTSUP if cuBLAS cannot be loaded. */
int ann_gemm_f32(ann_stream stream, const ann_view* a, const ann_view* b, const ann_view* c);
int ann_gemm_f64(ann_stream stream, const ann_view* a, const ann_view* b, const ann_view* c);

/* ---- qkvProjection: onHost/nn/attention.hpp:38-52 ---------------------- */
int ann_qkv_projection_f32(ann_stream stream, const ann_view* input, const ann_view* wq, const ann_view* wk,
                           const ann_view* wv, const ann_view* q, const ann_view* k, const ann_view* v);
int ann_qkv_projection_f64(ann_stream stream, const ann_view* input, const ann_view* wq, const ann_view* wk,
                           const ann_view* wv, const ann_view* q, const ann_view* k, const ann_view* v);

/* ---- outputProjection + residual: onHost/nn/attention.hpp:112-116 then
 * ops::add (onHost/ops/elementwise.hpp:307-311) -----------------------------
 * output = residual + input . Wo (row-major [N,K] x [K,M]); the add is the
 * cuBLAS epilogue (beta = 1), so the sum is rounded once instead of twice.
 * residual may be output. Throws on the gemm shape conditions or a residual
 * whose extents differ from output. */
int ann_output_projection_residual_f32(ann_stream stream, const ann_view* input, const ann_view* wo,
                                       const ann_view* residual, const ann_view* output);
int ann_output_projection_residual_f64(ann_stream stream, const ann_view* input, const ann_view* wo,
                                       const ann_view* residual, const ann_view* output);

/* ---- KV-cache append (one layer of an LBHTD cache, core/layout.hpp:41-45) --
 * The reference has no append kernel; its decode test fills the cache on the
 * host. k_new, v_new: BTHD [B,Tn,Hkv,D]; k_cache, v_cache: BHTD [B,Hkv,Tcap,D]
 * (for an LBHTD cache, the layer's sub-view). Writes the rows to cache tokens
 * [position, position + Tn). With cos/sin tables K is rotated on the way, with
 * the expression of ropeInPlace at positions position + t (bit-identical to
 * ropeInPlace followed by a plain append); cos = sin = NULL copies K as is.
 * Throws when the rows do not match the cache or do not fit its capacity. */
int ann_kv_cache_append_f32(ann_stream stream, const ann_view* k_new, const ann_view* v_new, const ann_view* k_cache,
                            const ann_view* v_cache, const ann_view* cos_table, const ann_view* sin_table,
                            uint32_t position);
int ann_kv_cache_append_f64(ann_stream stream, const ann_view* k_new, const ann_view* v_new, const ann_view* k_cache,
                            const ann_view* v_cache, const ann_view* cos_table, const ann_view* sin_table,
                            uint32_t position);

/* ---- elementwise ops: onHost/ops/elementwise.hpp ---------------------------
 * unaryOp / binaryOp over views of any rank and pitch with equal extents
 * (ANN_EINVAL "<op> shape mismatch." otherwise, elementwise.hpp:205-212).
 * Same expression order as the reference's operators, rounded per operation
 * (no fused multiply-add): copy/scale/add/sub/mul/div/axpy/relu/sqrt are
 * bit-identical to the reference's host arithmetic; exp, rsqrt, sigmoid,
 * silu, gelu and swiglu use the device math functions. In-place calls
 * (in == out) are allowed. */
#define ANN_UNARY_COPY 0    /* ops::copy            x                              */
#define ANN_UNARY_SCALE 1   /* ops::scale           x * scalar                     */
#define ANN_UNARY_EXP 2     /* ops::exp                                            */
#define ANN_UNARY_SQRT 3    /* ops::sqrt                                           */
#define ANN_UNARY_RSQRT 4   /* ops::rsqrt                                          */
#define ANN_UNARY_RELU 5    /* ops::relu            x > 0 ? x : 0                  */
#define ANN_UNARY_SIGMOID 6 /* ops::sigmoid         1 / (1 + exp(-x))              */
#define ANN_UNARY_SILU 7    /* ops::silu            x * sigmoid(x)                 */
#define ANN_UNARY_GELU 8    /* ops::gelu            0.5 * x * (1 + erf(x / sqrt 2)) */
int ann_unary_f32(ann_stream stream, int32_t op, const ann_view* in, const ann_view* out, float scalar);
int ann_unary_f64(ann_stream stream, int32_t op, const ann_view* in, const ann_view* out, double scalar);

#define ANN_BINARY_ADD 0    /* ops::add     l + r                      */
#define ANN_BINARY_SUB 1    /* ops::sub     l - r                      */
#define ANN_BINARY_MUL 2    /* ops::mul     l * r                      */
#define ANN_BINARY_DIV 3    /* ops::div     l / r                      */
#define ANN_BINARY_AXPY 4   /* ops::axpy    alpha * l + r              */
#define ANN_BINARY_SWIGLU 5 /* ops::swiglu  l * sigmoid(l) * r         */
int ann_binary_f32(ann_stream stream, int32_t op, const ann_view* lhs, const ann_view* rhs, const ann_view* out,
                   float alpha);
int ann_binary_f64(ann_stream stream, int32_t op, const ann_view* lhs, const ann_view* rhs, const ann_view* out,
                   double alpha);

/* ops::biasAdd (elementwise.hpp:348-366): out[..., h] = in[..., h] + bias[h],
 * bias 1-D with the extent of the last axis, then optionally an activation
 * in the same pass (nn::Activation, mlp.hpp:52-58): the result of biasAdd
 * followed by the activation in place, in one read and one write. */
#define ANN_ACT_NONE 0
#define ANN_ACT_RELU 1
#define ANN_ACT_SILU 2
#define ANN_ACT_GELU 3
int ann_bias_add_f32(ann_stream stream, const ann_view* in, const ann_view* bias, int32_t act, const ann_view* out);
int ann_bias_add_f64(ann_stream stream, const ann_view* in, const ann_view* bias, int32_t act, const ann_view* out);

/* ops::cast<T_Out> (elementwise.hpp:368-374) and ops::fill (:250-254): element
 * types by code; `value` points to one element of `dtype`. */
#define ANN_DTYPE_F32 0
#define ANN_DTYPE_F64 1
#define ANN_DTYPE_I32 2
#define ANN_DTYPE_U32 3
#define ANN_DTYPE_I64 4
int ann_cast(ann_stream stream, const ann_view* in, int32_t in_dtype, const ann_view* out, int32_t out_dtype);
int ann_fill(ann_stream stream, const ann_view* out, int32_t dtype, const void* value);

/* ---- axis reductions: onHost/ops/reduction.hpp ------------------------------
 * out has the input's rank and extents with extent 1 on `axis`
 * (validateReduction, reduction.hpp:173-188). Sums are formed in a different
 * order than the reference's sequential loop (within the reference tests'
 * 1e-5 / 1e-12); max is exact. mean divides by the axis extent. */
#define ANN_REDUCE_SUM 0
#define ANN_REDUCE_MAX 1
#define ANN_REDUCE_MEAN 2
#define ANN_REDUCE_SUM_SQUARES 3
#define ANN_REDUCE_DOT 4 /* ann_dot_* only */
int ann_reduce_f32(ann_stream stream, int32_t op, const ann_view* in, const ann_view* out, uint32_t axis);
int ann_reduce_f64(ann_stream stream, int32_t op, const ann_view* in, const ann_view* out, uint32_t axis);
/* ops::dot (reduction.hpp:259-283): sum over `axis` of lhs * rhs. */
int ann_dot_f32(ann_stream stream, const ann_view* lhs, const ann_view* rhs, const ann_view* out, uint32_t axis);
int ann_dot_f64(ann_stream stream, const ann_view* lhs, const ann_view* rhs, const ann_view* out, uint32_t axis);

/* ---- MLP layers: onHost/nn/mlp.hpp ------------------------------------------
 * Weights are row-major [in, out] (model format row_major_in_out), biases
 * 1-D [out]; activations ANN_ACT_*. GEMMs on cuBLAS; bias + activation in
 * one pass over the GEMM output.
 * linearBias (mlp.hpp:42-47) followed by an optional activation:
 * output = act(input . weight + bias). linear (:33-37) and decodeLatent
 * (:277-282) are ann_gemm_*. */
int ann_linear_bias_f32(ann_stream stream, const ann_view* input, const ann_view* weight, const ann_view* bias,
                        int32_t act, const ann_view* output);
int ann_linear_bias_f64(ann_stream stream, const ann_view* input, const ann_view* weight, const ann_view* bias,
                        int32_t act, const ann_view* output);
/* mlpForward (mlp.hpp:150-218): n_layers layers of
 * hidden = act(hidden . weights[l] + biases[l]), hidden_act on every layer but
 * the last, last_act on the last (the single-activation overload passes the
 * same value twice). Shape errors as the reference's, before anything is
 * enqueued. Scratch for the hidden activations: `workspace` of
 * workspace_bytes (ann_mlp_forward_workspace_bytes tells how many; 0 for one
 * layer), or NULL for a stream-ordered allocation on `stream`. */
int ann_mlp_forward_workspace_bytes(const ann_view* input, int32_t n_layers, const ann_view* weights,
                                    const ann_view* biases, const ann_view* output, size_t element_size,
                                    uint64_t* bytes);
int ann_mlp_forward_f32(ann_stream stream, const ann_view* input, int32_t n_layers, const ann_view* weights,
                        const ann_view* biases, int32_t hidden_act, int32_t last_act, const ann_view* output,
                        void* workspace, uint64_t workspace_bytes);
int ann_mlp_forward_f64(ann_stream stream, const ann_view* input, int32_t n_layers, const ann_view* weights,
                        const ann_view* biases, int32_t hidden_act, int32_t last_act, const ann_view* output,
                        void* workspace, uint64_t workspace_bytes);
/* mlp (mlp.hpp:307-337), the gated MLP:
 * output = swiglu(input . wgate, input . wup) . wdown. Scratch: two
 * [batch, hidden] buffers (2 * batch * hidden * element size bytes) in
 * `workspace`, or NULL for a stream-ordered allocation on `stream`. */
int ann_mlp_f32(ann_stream stream, const ann_view* input, const ann_view* wgate, const ann_view* wup,
                const ann_view* wdown, const ann_view* output, void* workspace, uint64_t workspace_bytes);
int ann_mlp_f64(ann_stream stream, const ann_view* input, const ann_view* wgate, const ann_view* wup,
                const ann_view* wdown, const ann_view* output, void* workspace, uint64_t workspace_bytes);

/* The gated MLP of ann_mlp_* for callers that cannot allocate device memory
 * while they run (a fixed memory budget, an allocator that must not be
 * re-entered). No counterpart in the reference, whose mlp allocates three
 * buffers per call. This call allocates nothing: the [batch, hidden]
 * activations go to a buffer that is part of the library image (8 MiB per
 * device, so batch * hidden * element size <= 8388608 bytes, else
 * ANN_EINVAL), and both GEMMs are the library's own kernels, not cuBLAS.
 * dtype: ANN_DTYPE_F32 or ANN_DTYPE_F64.
 * The 8 MiB are reserved when the CUDA runtime loads this code on a device:
 * under lazy module loading (CUDA 12's default, and what PyTorch sets) that is
 * the FIRST call on each device, so make that call at start-up, before a
 * memory budget is fixed and before any stream capture; later calls reserve
 * nothing, and the memory stays held until the process exits. The first call
 * on a device also looks up the buffer's address (cudaGetSymbolAddress) and
 * keeps it for that device for the life of the process; it does not survive a
 * cudaDeviceReset. Nothing in the buffer needs to start at zero. Calls whose
 * work overlaps on the GPU (different streams, no ordering) race on the
 * buffer. */
int ann_mlp_static_scratch(ann_stream stream, int32_t dtype, const ann_view* input, const ann_view* wgate,
                           const ann_view* wup, const ann_view* wdown, const ann_view* output);

/* ---- fused decode attention ----------------------------------------------
 * One launch computing the reference's decode pipeline
 *   attentionScores(q, k) -> ops::scale(scale) -> softmax(axis 3)
 *   -> attentionApply(probs, v)
 * (test/unit/nn/attention.cpp:675-734) without materialising scores/probs.
 * q, out: BTHD [B,Tq,Hq,D] (every query row attends to all Tk keys, the
 * non-causal softmax the reference uses for decode); k, v: `kv_layout` with
 * Tk keys and Hkv heads, query head hq reads kv head hq / g.
 * Requires unit innermost stride, 16-byte aligned K/V rows and Q rows, and
 * D in {64, 128, 256} (fp32) or {64, 128} (fp64); other shapes return
 * ANN_ENOTSUP (the per-op entry points above take any shape).
 * The key range of each row is split over the CTAs of one thread-block
 * cluster, merged in distributed shared memory: no workspace, no global
 * scratch memory. */
int ann_attention_decode_f32(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                             const ann_view* out, float scale, uint32_t queries_per_kv_group, int32_t kv_layout);
int ann_attention_decode_f64(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                             const ann_view* out, double scale, uint32_t queries_per_kv_group, int32_t kv_layout);

/* ---- fused prefill attention ---------------------------------------------
 * One launch computing the reference's prefill pipeline
 *   attentionScores(q, k) -> ops::scale(scale)
 *   -> causalSoftmax(axis 3, query axis 2, key axis 3)   (causal != 0)
 *      or softmax(axis 3)                               (causal == 0)
 *   -> attentionApply(probs, v)
 * (test/unit/nn/attention.cpp:591-651) without materialising scores/probs.
 * The causal mask is the reference's top-left one: key j is hidden from
 * query i iff i < j (onAcc/internal/nn/softmax.hpp:23-30), also when
 * Tq != Tk. q, out: BTHD [B,Tq,Hq,D]; k, v: `kv_layout` with Tk keys.
 * Requires unit innermost stride, 16-byte aligned rows, D in {64, 128}.
 * fp32 runs on the tensor cores (tcgen05 kind::tf32 with the 3xTF32 split,
 * fp32-level accuracy), by default on pairs of SMs that share every MMA
 * (cta_group::2); ANN_PREFILL_TC_PAIR=0 keeps one SM per CTA, and
 * ANN_PREFILL_FMA=1 selects the FP32-pipe kernel instead. fp64 runs on the
 * FP64 tensor cores (mma.sync m16n8k4.f64; ANN_PREFILL_FMA=1 selects the DFMA
 * kernel). */
int ann_attention_prefill_f32(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                              const ann_view* out, float scale, uint32_t queries_per_kv_group, int32_t kv_layout,
                              int32_t causal);
int ann_attention_prefill_f64(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                              const ann_view* out, double scale, uint32_t queries_per_kv_group, int32_t kv_layout,
                              int32_t causal);

/* ---- head sharding across the GPUs of one node ------------------------------
 * No reference counterpart: the reference path runs on one device. Attention
 * heads are independent (onAcc/internal/nn/attention.hpp:28-36, 57-64 read only
 * query head hq and KV head hq / g), so rank r of G computes heads
 * [r*H/G, (r+1)*H/G) and the per-rank output slabs are re-assembled with one
 * rank-major all-gather over NVLink. NCCL is loaded at first use; ANN_ENOTSUP
 * if libnccl.so.2 cannot be loaded.
 *
 * ann_comm_unique_id: rank 0 creates the rendezvous id and hands the
 *   ANN_COMM_ID_BYTES bytes to the other ranks out of band.
 * ann_comm_init: joins the communicator on the current CUDA device. Non-blocking:
 *   if the other ranks have not joined within timeout_s seconds, the half-built
 *   communicator is aborted and ANN_ENCCL returned. timeout_s is also the bound
 *   of the later calls on this communicator.
 * ann_comm_allgather: recv = the bytes_per_rank of every rank's send, rank-major,
 *   enqueued on `stream`.
 * ann_comm_destroy: flushes pending work (within the deadline, else aborts) and
 *   frees the communicator; ann_comm_abort tears it down at once (a peer died). */
int ann_comm_unique_id(unsigned char id[ANN_COMM_ID_BYTES]);
int ann_comm_init(ann_comm* comm, int32_t nranks, int32_t rank, const unsigned char id[ANN_COMM_ID_BYTES],
                  double timeout_s);
int ann_comm_size(ann_comm comm, int32_t* nranks, int32_t* rank);
int ann_comm_allgather(ann_comm comm, ann_stream stream, const void* send, void* recv, uint64_t bytes_per_rank);
int ann_comm_destroy(ann_comm comm);
int ann_comm_abort(ann_comm comm);

/* ---- head sharding without a collective: multicast ("mirror") outputs -------
 * No reference counterpart. The full output [B,T,H,D] lives in memory that
 * every rank of the node has bound to one NVLink multicast object (NVSwitch
 * NVLS; e.g. torch symmetric memory). Each rank computes its heads into its
 * slice `out` of its own copy, and `out_mirror` is the multicast address of
 * out's first element: every result store is a multimem store that the switch
 * writes into EVERY rank's copy, inside the producing kernel, so the gather
 * overlaps the computation tile by tile and needs neither a collective nor a
 * re-assembly pass. ann_signal_barrier, enqueued after them on every rank,
 * publishes all ranks' results to the rank's later work: it fences at system
 * scope before its release stores, which covers every store the producing
 * kernel made before it in stream order (the kernels themselves do not fence). Same shapes and semantics as
 * ann_attention_decode_* / ann_attention_prefill_* (prefill: the tensor-core
 * kernels only, else ANN_ENOTSUP). Only stores go through the multicast
 * address: nothing in this library loads from multicast or peer memory.
 *
 * ann_signal_barrier: `signals` = this rank's array of nranks uint32 words,
 *   zero before the first call; `peer_signals` = a DEVICE array of nranks
 *   pointers, entry p = rank p's array as addressed from this GPU (peer
 *   mappings; entry `rank` = signals). Stores `epoch` into word `rank` of every
 *   rank's array (release, system scope) and waits until every word of its
 *   own array holds it (acquire). Every rank calls it in the same order with
 *   epochs 1, 2, 3, ...; a wait that has not completed after timeout_ns sets
 *   ANN_DEVERR_WAIT_TIMEOUT (ann_take_device_error) and the kernel returns.
 *   nranks <= 32. Plain stores only: no multimem, no peer loads.
 * ann_signal_barrier_dev: the same barrier with the epoch kept in this rank's
 *   device memory: `epoch_word` (one uint32, zero before the first call) is
 *   read, its successor (skipping 0) used as the epoch and written back by the
 *   kernel, so the call can be captured in a CUDA graph and replayed. Use one
 *   of the two forms per signal array. */
int ann_attention_decode_mirror_f32(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                                    const ann_view* out, void* out_mirror, float scale,
                                    uint32_t queries_per_kv_group, int32_t kv_layout);
int ann_attention_decode_mirror_f64(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                                    const ann_view* out, void* out_mirror, double scale,
                                    uint32_t queries_per_kv_group, int32_t kv_layout);
int ann_attention_prefill_mirror_f32(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                                     const ann_view* out, void* out_mirror, float scale,
                                     uint32_t queries_per_kv_group, int32_t kv_layout, int32_t causal);
int ann_attention_prefill_mirror_f64(ann_stream stream, const ann_view* q, const ann_view* k, const ann_view* v,
                                     const ann_view* out, void* out_mirror, double scale,
                                     uint32_t queries_per_kv_group, int32_t kv_layout, int32_t causal);
int ann_signal_barrier(ann_stream stream, uint32_t* signals, uint32_t* const* peer_signals, int32_t nranks,
                       int32_t rank, uint32_t epoch, uint64_t timeout_ns);
int ann_signal_barrier_dev(ann_stream stream, uint32_t* signals, uint32_t* const* peer_signals, int32_t nranks,
                           int32_t rank, uint32_t* epoch_word, uint64_t timeout_ns);

/* ---- flat model artifacts: onHost/core/binary.hpp ------------------------
 * TensorSpec (binary.hpp:33-39): one tensor of a little-endian ".bin" file of
 * the neural-bunch model format v1. `shape` (row-major, informational) may be
 * NULL when shape_rank is 0. */
typedef struct ann_tensor_spec {
    const char* name;
    uint64_t offset_bytes;
    uint64_t count;
    const uint64_t* shape;
    int32_t shape_rank;
    int32_t reserved;
} ann_tensor_spec;

/* sha256File (binary.hpp:212-232): SHA-256 of the whole file as 64 lowercase
 * hex digits plus a NUL in hex_out. ANN_EIO if the file cannot be opened or
 * read. Host only, no device. */
int ann_sha256_file(const char* path, char hex_out[65]);
/* SHA-256 of a host buffer (the digest sha256File computes over a file). */
int ann_sha256_bytes(const void* data, size_t bytes, char hex_out[65]);

/* loadBinaryTensor<T> (binary.hpp:234-323), T = float (element_size 4) or
 * double (8): the spec's count elements at offset_bytes of `path` into
 * device_out (count * element_size bytes the caller allocated on the stream's
 * device, which must be current). Checks, in the reference's order and before
 * the payload is read: count != 0 (ANN_EINVAL); shape product == count
 * (ANN_EINVAL); the file can be stat'ed (ANN_EIO); offset_bytes % 64 == 0
 * (ANN_EINVAL); count * element_size does not overflow (ANN_EINVAL); the
 * byte range lies inside the file (ANN_EINVAL); when expected_sha256 is
 * non-empty, the file's digest equals it ignoring case (ANN_EIO). The copy is
 * enqueued on `stream`; the call returns once the payload has been read from
 * the file and handed to the copy engine (host staging is the library's).
 * device_out NULL: run the checks (digest included) and read nothing, so that
 * a wrapper can fail before it allocates, as the reference does. */
int ann_load_binary_tensor(ann_stream stream, const char* path, const ann_tensor_spec* spec, size_t element_size,
                           const char* expected_sha256, void* device_out);
/* One rank's rectangle of a tensor stored row-major as [rows, cols], rows =
 * spec->shape[0], cols = count / rows: rows [row_begin, row_begin+row_count)
 * x columns [col_begin, col_begin+col_count), written with a row pitch of
 * out_row_pitch_bytes. Loads a column-parallel (Wq/Wk/Wv) or row-parallel
 * (Wo) shard without reading the other ranks' columns. Same checks as
 * ann_load_binary_tensor, plus the box inside the tensor (ANN_EINVAL). The
 * reference loads whole tensors only. */
int ann_load_binary_tensor_box(ann_stream stream, const char* path, const ann_tensor_spec* spec,
                               size_t element_size, const char* expected_sha256, int64_t row_begin,
                               int64_t row_count, int64_t col_begin, int64_t col_count, void* device_out,
                               int64_t out_row_pitch_bytes);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* ANN_B200_H */
