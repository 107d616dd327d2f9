/*
 * kquant_oracle.h -- CPU restatement of the reference's K-quant hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may use it, and only as the checker.
 *
 * It restates, in plain scalar C, the algorithms of
 *   cpp/dequant_k.cpp      (block decoders, f16<->f32, the dequant_k export)
 *   cpp/moe_quant_dot.cpp  (quant_dot and the moe_quant_expert export)
 *   cpp/moe_delta.cpp      (the moe_delta_heads DeltaNet recurrence step)
 * of vin10122/Intel-optimized-MoE-streaming, including the reference's
 * 8-lane accumulation order, so that on the same host it reproduces the
 * reference library bit for bit.  The block formats themselves are those of
 * gguf-py 0.19.0 (gguf.quants), the third-party package the reference pins
 * its dequant results against (tools/test_dequant_k.py:121).
 */
#ifndef KQUANT_ORACLE_H
#define KQUANT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    KQ_Q8_0 = 8,
    KQ_Q3_K = 11,
    KQ_Q4_K = 12,
    KQ_Q5_K = 13,
    KQ_Q6_K = 14,
};

float    kq_f16_to_f32(uint16_t h);
uint16_t kq_f32_to_f16(float f);
float    kq_round16(float f);

int kq_block_size(int type);
int kq_block_bytes(int type);

/* One block -> block_size floats, same bits as the reference decoders. */
int kq_dequant_block(int type, const uint8_t* blk, float* out);

/* Same contract as the reference export dequant_k (cpp/dequant_k.cpp:350). */
int kq_dequant(int type, const uint8_t* src, void* dst, int64_t n, int want_f16);

/* One quantised row dotted with x, reference lane order (moe_quant_dot.cpp:143). */
float kq_quant_dot(int type, const uint8_t* row, const float* x, int columns,
                   int round_weights);

/* Same contract as the reference export moe_quant_expert
   (cpp/moe_quant_dot.cpp:171-214), status codes included. */
int kq_expert(int gate_type, const uint8_t* gate, int64_t gate_bytes,
              int up_type, const uint8_t* up, int64_t up_bytes,
              int down_type, const uint8_t* down, int64_t down_bytes,
              const float* input, int hidden, int intermediate, float* output,
              int fp16_graph);

/* Same contract as the reference export moe_delta_heads
   (cpp/moe_delta.cpp:18-69): one gated delta-rule step over every head's
   fp32 state, in place, status codes and early stop included. */
int kq_delta_heads(float* state, const float* q, const float* k,
                   const float* v, const float* beta, const float* gate,
                   float* output, int heads, int key_dim, int value_dim);

#ifdef __cplusplus
}
#endif
#endif
