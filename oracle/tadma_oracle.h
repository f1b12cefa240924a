/*
 * tadma_oracle.h - CPU restatement of TADMA's tensor-library hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker that the CUDA library is
 * compared against; nothing in the product (tadma_b200/, include/) links,
 * imports or calls it.  Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline / reference legs use it.
 *
 * PARITY UNPINNED: the reference (OgnianM/TADMA) needs clang >= 19 / C++23
 * (deducing-this, pack indexing) and cannot be compiled or run in this image,
 * and it ships no tests or golden vectors.  This restatement follows the
 * reference source line by line (citations per function, paths relative to
 * the reference project root) and is pinned only by analytic known-answer
 * tests (tests/golden/).
 *
 * Tensor descriptors are the C-ABI's tadma_tensor with HOST pointers.
 */
#ifndef TADMA_ORACLE_H
#define TADMA_ORACLE_H

#include <stdint.h>
#include "../include/tadma_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* scalar conversions (round to nearest even) */
uint16_t or_f32_to_f16(float f);
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_bf16(float f);
float or_bf16_to_f32(uint16_t h);
uint16_t or_f64_to_f16(double v);  /* one rounding, no detour through fp32 */
uint16_t or_f64_to_bf16(double v);

/* seeded generator (same definition as tadma_b200_fill) */
uint64_t or_mix64(uint64_t z);
int or_fill(const tadma_tensor* out, int32_t dist, double p0, double p1, uint64_t seed,
            uint64_t stream_id, int64_t offset);
/* The standard normal value of global element g (before mean / std / rounding). */
double or_gen_normal(uint64_t seed, uint64_t stream_id, uint64_t g);

/* MapToShape (include/tadma/Utils.hpp:9-17): linear -> row-major multi-index */
void or_map_to_shape(const int64_t* dims, int32_t rank, int64_t index, int64_t* out_idx);

/* generic ops, same contracts as the C ABI entry points */
int or_eltwise(const tadma_tensor* out, const tadma_tensor* ins, int32_t n_ins,
               const tadma_instr* prog, int32_t n_instr, int32_t compute);
int or_reduce(int32_t op, const tadma_tensor* in, int32_t axis, int32_t pre_op,
              const tadma_tensor* out);
int or_softmax(const tadma_tensor* in, int32_t axis, const tadma_tensor* out);
int or_layer_norm(const tadma_tensor* in, int32_t axis, const tadma_tensor* gamma,
                  const tadma_tensor* beta, double eps, int32_t mode, const tadma_tensor* out);
int or_rms_norm(const tadma_tensor* in, int32_t axis, double eps, const tadma_tensor* out);
int or_gather(const tadma_tensor* table, int32_t axis, const tadma_tensor* ids,
              const tadma_tensor* add, const tadma_tensor* out);

/* straightforward per-config host loops (the timed CPU baseline), OpenMP over rows */
void or_cfg2_gelu_affine_bf16(const uint16_t* x, const uint16_t* bias, float s, uint16_t* y,
                              int64_t rows, int64_t cols);
/* Row reductions in the reference's own ReduceKernel fold order and
 * accumulator type (fp32, or fp16 in fp16): op 0 sum, 1 max, 2 mean. */
int or_reduce_rows_reference_order(int32_t op, const void* x, int32_t dtype, int64_t rows, int64_t R, void* out);
void or_cfg3_sum_lastaxis_f32(const float* x, float* y, int64_t rows, int64_t cols);
void or_cfg3_max_lastaxis_f32(const float* x, float* y, int64_t rows, int64_t cols);
void or_cfg3_argmax_lastaxis_f32(const float* x, int64_t* y, int64_t rows, int64_t cols);
void or_cfg3_mean_midaxis_f32(const float* x, float* y, int64_t outer, int64_t r, int64_t inner);
void or_cfg4_layer_norm_f16(const uint16_t* x, const uint16_t* g, const uint16_t* b, double eps,
                            uint16_t* y, int64_t rows, int64_t cols);
void or_cfg4_softmax_f16(const uint16_t* x, uint16_t* y, int64_t rows, int64_t cols);
void or_cfg5_gather_add(const uint16_t* table_f16, int64_t vocab, const int64_t* ids,
                        const uint16_t* pos_bf16, uint16_t* out_bf16, int64_t batch,
                        int64_t seq, int64_t dim);

int or_num_threads(void);
void or_set_num_threads(int n);

#ifdef __cplusplus
}
#endif

#endif
