/*
 * moe_b200.h -- C ABI of libmoe_b200.so, the B200 (sm_100a) routed-expert
 * MoE library.
 *
 * Two groups of entry points:
 *
 * 1. Drop-ins for the reference's native exports.  Same names, argument
 *    meaning, return codes and synchronous behaviour as the functions of
 *    vin10122/Intel-optimized-MoE-streaming that Python binds with ctypes.
 *    Pointers may be host memory (copied to the GPU and back inside the
 *    call) or device memory (used in place).  The calling thread's current
 *    CUDA device is used.
 *
 * 2. A device-resident API: weights stay in HBM in their GGUF block layout,
 *    every pointer is a device pointer, every call is asynchronous on the
 *    given cudaStream_t (passed as void*), and argument errors are returned
 *    before anything is enqueued.
 *
 * Status codes (all functions returning int): 0 success;
 *   -1 bad argument (null pointer, size <= 0 or out of range, bad flag),
 *   -2 unsupported ggml type or columns not a multiple of its block size
 *      (moe_delta_heads: an output is not finite, the reference's meaning),
 *   -3 tensor byte count does not match its shape,
 *   -4 an output value is not finite,
 *   -5 host-side failure (allocation),
 * and, for conditions the CPU reference cannot have,
 *   -6 a CUDA call failed (moe_b200_last_cuda_error() gives the cudaError_t),
 *   -7 a device pointer is not 16-byte aligned (4-byte for the DeltaNet step),
 *   -8 workspace too small,
 *   -9 a bounded device-side wait gave up.
 *
 * ggml type ids: Q8_0 = 8, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14.
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_B200_API __attribute__((visibility("default")))
#else
#define MOE_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * 1. Reference-compatible exports
 * ---------------------------------------------------------------------- */

/* 1 if `type` is one of the five supported ggml types, else 0.
 * Replaces dequant_k_supported (cpp/dequant_k.cpp:342-344). */
MOE_B200_API int dequant_k_supported(int type);

/* Values per block of `type` (32 or 256), 0 if unsupported.
 * Replaces dequant_k_block_size (cpp/dequant_k.cpp:346-348). */
MOE_B200_API int dequant_k_block_size(int type);

/* Dequantise n values of `type` from src into dst: fp32, or binary16
 * rounded to nearest even when want_f16 != 0.  Bit-identical to the
 * reference.  Returns 0, or -1 on an unknown type, a null pointer, n <= 0 or
 * n not a multiple of the block size (-6 on a CUDA failure).
 * Replaces dequant_k (cpp/dequant_k.cpp:350-394); bound by ctypes in
 * src/run_q4k_f16_openvino.py:37-59 and tools/test_dequant_k.py:52-76. */
MOE_B200_API int dequant_k(int type, const uint8_t* src, void* dst, int64_t n, int want_f16);

/* One SwiGLU expert for one token over raw quantised rows:
 *   g = gate.x, u = up.x, a = (g * sigmoid(g)) * u, output = down.a
 * gate/up are [intermediate x hidden], down is [hidden x intermediate], each
 * a row-major sequence of GGUF blocks.  fp16_graph = 1 rounds x, every
 * weight, g, u, sigmoid, silu, a and the output to binary16 like the
 * reference; 0 computes in fp32.  Status codes as listed above, checked in
 * the reference's order; on -4 the rows after the first non-finite one are
 * left untouched.
 * Replaces moe_quant_expert (cpp/moe_quant_dot.cpp:171-214); bound by
 * ctypes in src/flash_moe/native_expert.py:14-20. */
MOE_B200_API int moe_quant_expert(int gate_type, const uint8_t* gate, int64_t gate_bytes,
                     int up_type, const uint8_t* up, int64_t up_bytes,
                     int down_type, const uint8_t* down, int64_t down_bytes,
                     const float* input, int hidden, int intermediate, float* output,
                     int fp16_graph);

/* One gated delta-rule (DeltaNet) decode step over every head, in place on
 * the fp32 state [heads][value_dim][key_dim]:
 *   decay = exp(double(gate[h])); row <- float(double(row) * decay);
 *   kv = row . k[h]; delta = beta[h] * (v[h][r] - kv);
 *   row <- row + delta * k[h]; output[h][r] = row . q[h]
 * with q, k [heads][key_dim], v and output [heads][value_dim], beta and gate
 * [heads].  Sums in the reference's eight-lane order: bit-identical to it.
 * Returns 0; -1 for a null pointer, heads outside 1..256 or key_dim,
 * value_dim outside 1..1024; -2 when an output is not finite.  On -2, as in
 * the reference, rows up to and including the first non-finite one hold
 * their new state and outputs are written only for the rows before it; a
 * state in host memory keeps its later rows unchanged, a state in device
 * memory has every row updated.  -9 when a bounded device-side wait gave up.
 * Any pointer may be host or device memory.
 * Replaces moe_delta_heads (cpp/moe_delta.cpp:18-69); bound by ctypes in
 * src/flash_moe/native_expert.py:76-98 (NativeDelta) and called from
 * src/flash_moe/gated_deltanet.py:386. */
MOE_B200_API int moe_delta_heads(float* state, const float* q, const float* k, const float* v,
                                 const float* beta, const float* gate, float* output, int heads,
                                 int key_dim, int value_dim);

/* ------------------------------------------------------------------------
 * 2. Device-resident API
 * ---------------------------------------------------------------------- */

/* One MoE layer resident in device memory.  Routed-expert tensors are the
 * GGUF ffn_{gate,up,down}_exps tensors (or the slice of them this GPU holds):
 * `expert_count` consecutive per-expert tensors, expert e (global id) at
 * byte offset (e - expert_begin) * per-expert size.  Base pointers must be
 * 16-byte aligned.  Replaces the per-expert byte ranges the reference slices
 * out of the GGUF file (src/run_q4k_f16_openvino.py:88-133) and keeps them
 * resident instead of streaming them (src/flash_moe/store.py:138-239). */
typedef struct moe_b200_layer {
    int32_t hidden;              /* H */
    int32_t intermediate;        /* I of the routed experts */
    int32_t n_experts;           /* E: experts the router scores */
    int32_t top_k;               /* K, 1..16 */
    int32_t expert_begin;        /* first expert held in gate/up/down */
    int32_t expert_count;        /* experts held (E when not sharded) */
    int32_t gate_type, up_type, down_type;
    int32_t shared_intermediate; /* 0: no shared expert */
    int32_t shared_gate_type, shared_up_type, shared_down_type;
    int32_t flags;               /* MOE_B200_* flags below */
    const uint8_t* gate;         /* expert_count x [I x H] blocks */
    const uint8_t* up;           /* expert_count x [I x H] blocks */
    const uint8_t* down;         /* expert_count x [H x I] blocks */
    const float* router;         /* [E x H] fp32, the GGUF ffn_gate_inp layout */
    const float* router_bias;    /* [E] fp32 added to the logits, or NULL */
    const uint8_t* shared_gate;  /* [Is x H] */
    const uint8_t* shared_up;    /* [Is x H] */
    const uint8_t* shared_down;  /* [H x Is] */
    const float* shared_gate_inp;/* [H] fp32 */
} moe_b200_layer;

/* flags */
#define MOE_B200_FP16_GRAPH   1  /* routed experts with the fp16_graph rounding */
#define MOE_B200_NO_SHARED    2  /* skip the shared expert on this call */
#define MOE_B200_EXACT        4  /* use the exact (fp32 dequant + FMA) engine */
#define MOE_B200_SHARED_ONLY  8  /* only the shared expert (no routing, no routed experts) */
#define MOE_B200_TCGEN05     16  /* prefill: the tcgen05 expert GEMMs also for <= 48 tokens */

/* Bytes of workspace moe_b200_decode needs for `max_tokens` tokens.  The
 * workspace is 256-byte aligned device memory; zero it once with
 * moe_b200_workspace_init before its first use.  Calls sharing one
 * workspace must be ordered (same stream). */
MOE_B200_API int moe_b200_decode_workspace(const moe_b200_layer* layer, int32_t max_tokens,
                              size_t* bytes);

/* Decode `tokens` tokens through one layer, all on `stream`:
 *   route (fp32 scores, top-k, float64 softmax over the k) ->
 *   k routed SwiGLU experts -> sum of weight_k * out_k in top-k order ->
 *   + sigmoid(x . shared_gate_inp) * shared_expert(x).
 * x: [tokens x H] fp32, y: [tokens x H] fp32.  topk_ids ([tokens x K]
 * int32) and topk_weights ([tokens x K] fp32) receive the routing when not
 * NULL.  Experts outside [expert_begin, expert_begin + expert_count)
 * contribute zero (expert-parallel partial output).
 * Replaces run_moe_layer (src/flash_moe/moe_layer.py:39-107) with the
 * router of src/flash_moe/router.py:140-170 and the shared expert of
 * src/flash_moe/shared_expert.py:221-251, for each token. */
MOE_B200_API int moe_b200_decode(const moe_b200_layer* layer, const float* x, int32_t tokens,
                    float* y, int32_t* topk_ids, float* topk_weights,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace moe_b200_decode_host needs for `max_tokens` tokens:
 * the decode workspace plus device staging rows for x, y and the routing. */
MOE_B200_API int moe_b200_decode_host_workspace(const moe_b200_layer* layer, int32_t max_tokens,
                                   size_t* bytes);

/* moe_b200_decode for a caller whose token rows and results live in HOST
 * memory, synchronous like the reference's ctypes entry points: copies x
 * ([tokens x H] fp32) to the workspace's staging rows, decodes on `stream`,
 * copies y (and topk_ids / topk_weights when not NULL) back to the host
 * pointers and waits for the stream.  One token goes through this calling
 * thread's pinned staging rows (allocated on its first call, kept until the
 * process exits) and one graph launch whose kernels read the token and write
 * the result through the pinned mapping; several tokens are copied with
 * cudaMemcpyAsync (pinned rows make those copies asynchronous).  Returns
 * moe_b200_decode's status, or -9 when a bounded device wait gave up (the
 * workspace error word, read and cleared here).  The workspace is device
 * memory of moe_b200_decode_host_workspace bytes, zeroed once with
 * moe_b200_workspace_init.  This is the host-side form of run_moe_layer
 * (src/flash_moe/moe_layer.py:39-107), whose activations and outputs are
 * numpy arrays: one call per layer instead of one moe_quant_expert call per
 * selected expert (src/flash_moe/native_expert.py:23-37). */
MOE_B200_API int moe_b200_decode_host(const moe_b200_layer* layer, const float* x, int32_t tokens,
                         float* y, int32_t* topk_ids, float* topk_weights,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Zero the whole workspace (`workspace_bytes`) on `stream`.  Call once
 * after allocating a decode workspace, before its first use.  The decode
 * kernels leave the counters zero again when they finish; the fused
 * single-token kernel also keeps a step sequence number there that tags the
 * values its CTAs exchange, so zeroing only part of a workspace that has
 * been used could let a stale value pass as a current one. */
MOE_B200_API int moe_b200_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Synchronously read (and clear) the device-side error word of a
 * workspace: 0; -9 when a bounded wait of a decode or prefill launch gave
 * up; -10 when a prefill SwiGLU activation fell outside the fp16 range
 * (that call's output is not valid; moe_b200_decode computes the same
 * tokens in fp32). */
MOE_B200_API int moe_b200_workspace_error(void* workspace, void* stream, int* error);

/* Number of kernels one moe_b200_decode call with this layer, token count
 * and the layer's flags launches (1 for the fused paths: one token, or up
 * to 8 tokens and SHARED_ONLY calls of up to 8 tokens). */
MOE_B200_API int moe_b200_decode_kernels(const moe_b200_layer* layer, int32_t tokens,
                                         int* kernels);

/* Many-token layer forward on the tcgen05 tensor cores: the prefill form of
 * run_moe_sequence (reference src/flash_moe/moe_layer.py:110-195, whose
 * per-expert batches go through ExpertBackend.forward_batch,
 * src/flash_moe/backend_ov.py:357-431, and SharedExpert.forward_batch,
 * src/flash_moe/shared_expert.py:200-219).  No single reference function
 * has this signature: it is the device-resident prefill export the B200
 * library adds beside the per-expert ones.
 *
 * x: device [tokens x hidden], fp32 (x_dtype 0) or bf16 (x_dtype 1).
 * y: device fp32 [tokens x hidden], written in full.  topk_ids /
 * topk_weights: device [tokens x top_k] or NULL.  The expert weights are
 * dequantised to fp16 (the value of dequant_k with want_f16 = 1) and the
 * products accumulate in fp32; the result matches the fp32 reference
 * within 1e-3 relative (max |y - ref| / max |ref|).  Flags: NO_SHARED and
 * SHARED_ONLY as for moe_b200_decode; EXACT and FP16_GRAPH are not
 * available here (-2).  Returns -2 when a shape or block format is outside
 * this path (moe_b200_prefill_supported), -8 for a short workspace.
 * Asynchronous on `stream`; calls sharing a workspace must be ordered on
 * one stream. */
MOE_B200_API int moe_b200_prefill(const moe_b200_layer* layer, const void* x, int32_t x_dtype,
                                  int32_t tokens, float* y, int32_t* topk_ids,
                                  float* topk_weights, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* Workspace bytes of moe_b200_prefill for up to max_tokens tokens (device
 * memory, 256-byte aligned; its first 256 bytes are the control words;
 * moe_b200_workspace_init zeroes it before first use). */
MOE_B200_API int moe_b200_prefill_workspace(const moe_b200_layer* layer, int32_t max_tokens,
                                            size_t* bytes);

/* 1 when moe_b200_prefill handles this layer and its flags: hidden,
 * intermediate and shared_intermediate multiples of 256, hidden at most
 * 8192; Q8_0, Q3_K, Q4_K, Q5_K or Q6_K weights whose rows are multiples of
 * 16 bytes; gate and up of one format; at most 1024 held experts. */
MOE_B200_API int moe_b200_prefill_supported(const moe_b200_layer* layer);

/* Number of kernels one moe_b200_prefill call of `tokens` tokens launches
 * (7; for at most 128 tokens, whose router runs on the CUDA cores, 5 with at
 * most 256 experts -- the router also selects the top-k -- else 6; 3 with
 * MOE_B200_SHARED_ONLY). */
MOE_B200_API int moe_b200_prefill_kernels(const moe_b200_layer* layer, int tokens, int* kernels);

/* One step of a multi-step decode launch (moe_b200_decode_steps). */
typedef struct moe_b200_step {
    int32_t layer;            /* index into the layer table */
    int32_t flags;            /* MOE_B200_STEP_* */
    const float* x;           /* device [hidden] token (not read with CHAIN) */
    float* y;                 /* device [hidden] output */
    int32_t* topk_ids;        /* device [top_k] or NULL */
    float* topk_weights;      /* device [top_k] or NULL */
} moe_b200_step;

#define MOE_B200_STEP_CHAIN 1 /* the input is the previous step's output */
#define MOE_B200_STEP_BLOCK 2 /* transformer block with an identity mixer:
                                 h = x + rmsnorm16(x), y = h + f16(MoE(rmsnorm16(h))),
                                 RMSNorm weight 1 (src/flash_moe/transformer.py:229-247,
                                 norm.py:21-30) */

/* n_steps single-token layer steps in ONE cooperative launch of the fused
 * decode kernel: the whole decode of a token through a stack of layers
 * (CHAIN | BLOCK steps), or independent tokens.  No reference function has
 * this signature: it replaces the per-layer loop of Qwen3MoEModel.forward
 * (src/flash_moe/model.py) over run_moe_layer (moe_layer.py:39-107) for a
 * decode step.  layer0 (host) gives the shapes and block formats that every
 * layer of the device table layers_dev shares, and the flags (NO_SHARED
 * allowed); steps_dev is a device array of n_steps entries.  The workspace
 * is the one moe_b200_decode_workspace(layer0, 1, ...) sizes.  Returns -2
 * when the fused kernel does not take these shapes or formats. */
MOE_B200_API int moe_b200_decode_steps(const moe_b200_layer* layer0,
                                       const moe_b200_layer* layers_dev,
                                       const moe_b200_step* steps_dev, int32_t n_steps,
                                       float eps, void* workspace, size_t workspace_bytes,
                                       void* stream);

/* One rank's part of an expert-parallel decode step over the tokens of
 * all ranks (x: [tokens x H], tokens <= 8), in one cooperative launch:
 * route every token with the replicated router, add the outputs of the
 * selected experts this rank holds (expert_begin / expert_count), and add
 * the sigmoid-gated shared expert to tokens [shared_begin, shared_begin +
 * shared_count) only -- the rank's own tokens -- so that the sum of the
 * partial outputs y over the ranks (the combine) is each token's layer
 * output with the shared expert counted once.  No reference function has
 * this signature: it replaces run_moe_layer (src/flash_moe/moe_layer.py:
 * 39-107) on the expert-sharded layer.  Flags NO_SHARED / SHARED_ONLY are
 * not accepted (-1); returns -2 when the fused multi-token kernel does not
 * take these shapes or formats.  Workspace as moe_b200_decode_workspace
 * with max_tokens >= tokens. */
MOE_B200_API int moe_b200_decode_ep(const moe_b200_layer* layer, const float* x, int32_t tokens,
                                    int32_t shared_begin, int32_t shared_count, float* y,
                                    int32_t* topk_ids, float* topk_weights, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* Expert-parallel decode with the dispatch and the combine inside the
 * layer kernel, over NVLink peer memory instead of collectives.  Each rank
 * creates an exchange context (device buffer for the gathered tokens, the
 * partial outputs and the step flags), publishes its blob of
 * MOE_B200_EP_BLOB_BYTES bytes (an IPC handle and the agreed shape), and
 * connects with the blobs of all ranks in rank order.  Every rank must have
 * the same world, tokens_per_rank, hidden and multiprocessor count.
 * moe_b200_decode_ep_p2p then runs one step: it pushes this rank's x
 * [tokens_per_rank x H] to every rank, routes all world * tokens_per_rank
 * tokens, applies the experts this rank holds, pushes each token's partial
 * output to its owner, and writes into y the sum over ranks (rank order) for
 * this rank's tokens, with the shared expert added once by the owner.
 * Every rank runs the same steps in the same order; a rank that waits
 * longer than about a second for its peers records -9 in the workspace
 * error word.  topk_ids / topk_weights ([world * tokens_per_rank x K])
 * receive the routing of every gathered token (row r * tokens_per_rank + j:
 * rank r's token j).  No reference function has these signatures: they
 * replace the per-layer run_moe_layer call (src/flash_moe/moe_layer.py:
 * 39-107) of an expert-sharded model. */
#define MOE_B200_EP_BLOB_BYTES 128
typedef struct moe_b200_ep moe_b200_ep;
MOE_B200_API int moe_b200_ep_create(int32_t world, int32_t rank, int32_t tokens_per_rank,
                                    int32_t hidden, moe_b200_ep** ctx, void* blob);
MOE_B200_API int moe_b200_ep_connect(moe_b200_ep* ctx, const void* blobs);
MOE_B200_API int moe_b200_ep_destroy(moe_b200_ep* ctx);
MOE_B200_API int moe_b200_decode_ep_p2p(const moe_b200_layer* layer, moe_b200_ep* ctx,
                                        const float* x, float* y, int32_t* topk_ids,
                                        float* topk_weights, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* The transformer block with an identity mixer around a many-token MoE
 * call, for T tokens of H values (device fp32, row-major):
 *   moe_b200_block_prepare: h = x + f16(rmsnorm(x)), n = f16(rmsnorm(h))
 *   moe_b200_block_finish:  y = h + f16(m), m the MoE output of n
 * RMSNorm with weight 1: v / sqrt(mean(v^2) + eps) (src/flash_moe/norm.py:21-30;
 * the block, src/flash_moe/transformer.py:229-247).  Single-token stacks run
 * the same block inside moe_b200_decode_steps (MOE_B200_STEP_BLOCK). */
MOE_B200_API int moe_b200_block_prepare(const float* x, float* h, float* n, int32_t tokens,
                                        int32_t hidden, float eps, void* stream);
MOE_B200_API int moe_b200_block_finish(const float* h, const float* m, float* y, int32_t tokens,
                                       int32_t hidden, void* stream);

/* Largest `intermediate` moe_b200_expert_noalloc accepts. */
#define MOE_B200_NOALLOC_MAX_INTERMEDIATE 16384

/* moe_quant_expert for callers that cannot allocate device memory -- a
 * serving process that reserved all of it up front for its own pool, or a
 * thread that must not enter the CUDA allocator while other work runs
 * (freeing, and allocating when memory has to be returned first,
 * synchronise the device).  No counterpart in the reference.
 *
 * Same arguments, arithmetic and argument checks as moe_quant_expert, but
 * every pointer must be device memory (input and output 16-byte aligned),
 * the call is asynchronous on `stream` (a cudaStream_t), and it allocates
 * nothing: its scratch (the intermediate activations) is a fixed array
 * inside the library, 2 x MOE_B200_NOALLOC_MAX_INTERMEDIATE floats that
 * every GPU loading the library holds until the process exits.  Returns -1
 * also when intermediate exceeds MOE_B200_NOALLOC_MAX_INTERMEDIATE.  A
 * non-finite output is not reported (use moe_quant_expert for status -4).
 * The first call on a device looks up the array's device address (once per
 * device); make that first call before any stream capture.  All calls on a
 * device share the array: calls whose kernels overlap on the GPU race, so
 * order them on one stream. */
MOE_B200_API int moe_b200_expert_noalloc(int gate_type, const uint8_t* gate, int64_t gate_bytes,
                                         int up_type, const uint8_t* up, int64_t up_bytes,
                                         int down_type, const uint8_t* down, int64_t down_bytes,
                                         const float* input, int hidden, int intermediate,
                                         float* output, int fp16_graph, void* stream);

/* moe_delta_heads on device pointers, asynchronous on `stream` (no host
 * synchronisation, capturable in a CUDA graph).  decay = exp(double(gate))
 * is computed on the device (CUDA's double exp: the decayed state can differ
 * from the host entry point's in the last bit of a float, rarely).  Every
 * row is updated and every output written.  status (device int32[2], may be
 * NULL) receives in [0] -1, or the smallest flat row index h * value_dim + r
 * whose output is not finite, and in [1] 0, or nonzero when a bounded
 * device-side wait gave up (the state is then partly updated).  Returns 0,
 * -1 (arguments, as above), -7 for a pointer that is not 4-byte aligned, -6
 * on a CUDA launch failure. */
MOE_B200_API int moe_b200_delta_heads(float* state, const float* q, const float* k,
                                      const float* v, const float* beta, const float* gate,
                                      float* output, int heads, int key_dim, int value_dim,
                                      int32_t* status, void* stream);

/* Device-pointer dequantisation on a stream: out_dtype 0 = fp32,
 * 1 = binary16 (round to nearest even).  Same values as dequant_k. */
MOE_B200_API int moe_b200_dequant(int type, const void* src, void* dst, int64_t n, int out_dtype,
                     void* stream);

/* Phase tracing of the fused decode kernel: while set, every fused launch
 * from this thread writes, per CTA c, 32 uint64 global-timer stamps (ns)
 * to device_buffer[32 * c ...] at its phase boundaries (0 entry, 1 token
 * quantised, 2 first copies landed, 3 router done, 4 shared gate/up done,
 * 5 routing known, 6 top-k done, 7 routed gate/up done, 8 after barrier,
 * 9 all activations published, 10 down inputs ready, 11 down done, 12 exit;
 * 13-15 inside the top-k, 16-22 inside the routed and down phases).  capacity_ctas must cover the grid (one CTA
 * per SM).  NULL switches tracing off. */
MOE_B200_API int moe_b200_set_trace(void* device_buffer, int capacity_ctas);

/* cudaError_t of the last failed CUDA call on this thread (0 if none). */
MOE_B200_API int moe_b200_last_cuda_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
MOE_B200_API int moe_b200_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
