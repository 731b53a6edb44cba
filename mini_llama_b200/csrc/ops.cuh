// ops.cuh — small device ops (host-side launchers).
#pragma once

#include "common.cuh"

namespace mlb {

void op_rmsnorm(const float* x, const float* w, int n, float eps, float* y, cudaStream_t s);
void op_silu(const float* x, int n, float* y, cudaStream_t s);
void op_mul(const float* a, const float* b, int n, float* y, cudaStream_t s);
void op_add(const float* a, const float* b, int n, float* y, cudaStream_t s);
void op_softmax(const float* x, int n, float* y, cudaStream_t s);
void op_embedding(const float* table, int vocab, int dim, const int* token_dev, int token_host,
                  float* y, cudaStream_t s, bool pdl);
void op_rope(float* q, float* k, int nh, int nkv, int D, int neox, const float2* cs_dev,
             cudaStream_t s);
void op_kv_write(float* keys, float* values, size_t slot, int n, const float* k, const float* v,
                 cudaStream_t s);
void op_argmax(const float* x, int n, int* out_dev, int* out_dev2, cudaStream_t s, bool pdl);
void op_fill(float* p, long long n, float v, cudaStream_t s);
void rope_table_host(float theta, int D, int pos0, int npos, float2* out);
// Seeded GGUF blocks for destination rows whose source rows are src_rows[i]
// (-1 = zero row), or row0 + i when src_rows is null.
void synth_gguf_blocks_rows(int qtype, uint64_t key, float scale, int raw, long long row0,
                            long long rows, long long blk0, long long nblk, long long full_cols,
                            const int* src_rows, uint8_t* dst, size_t dst_pitch,
                            cudaStream_t stream);

}  // namespace mlb
