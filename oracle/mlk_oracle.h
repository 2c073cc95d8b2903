/* CPU restatement of the reference buffer executor (test infrastructure
 * only; see mlk_oracle.c). */
#ifndef MLK_ORACLE_H
#define MLK_ORACLE_H
#include <stdint.h>
#include "../include/mlkb200.h"
#ifdef __cplusplus
extern "C" {
#endif
int mlko_chain(int32_t n_roots, const int32_t* root_len, const mlkb_expr* exprs,
               int32_t poly7, const double* a, const double* b, double* const* outs,
               int64_t n, const double* scalars, int64_t n_scalars);
int mlko_softmax(const double* a, double* y, int64_t rows, int64_t cols);
int mlko_reducesum(const double* a, double* y, int64_t rows, int64_t cols);
int mlko_matmul_rows(const double* a, const double* b, double* c, int64_t n,
                     int64_t k, int64_t row_begin, int64_t row_end);
int mlko_matmul(const double* a, const double* b, double* c, int64_t m,
                int64_t n, int64_t k);
uint64_t mlko_word(uint64_t seed, uint32_t stream_id, uint64_t i);
void mlko_fill_uniform_f32(float* out, int64_t n, uint64_t seed,
                           uint32_t stream_id, double lo, double hi, int64_t first);
#ifdef __cplusplus
}
#endif
#endif
