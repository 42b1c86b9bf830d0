// Decode-step kernels of the tensor-parallel Llama model (nab_llama.cu).
#pragma once

#include <cuda_runtime.h>

namespace nab {

// Rotary embedding of q and k (head_dim 128, half-split convention) and append
// of k, v at position *pos of the caches [B, Hkv, Lmax, 128].
void rope_append(cudaStream_t s, const void* qkv, const float* cos_t, const float* sin_t, const int* pos,
                 void* q_out, void* k_cache, void* v_cache, int B, int Hq, int Hkv, int Lmax);

// GQA decode attention over positions [0, *pos] of the cache, q [B, Hq, 128]
// (already rotated). splits in [1, 16] CTAs per (batch, kv head), combined
// in the same launch; no scratch.
void decode_attention(cudaStream_t s, const void* q, const void* k_cache, const void* v_cache, const int* pos,
                      void* out, int B, int Hq, int Hkv, int Lmax, int splits);
// RoPE + KV append + attention in one launch, from the qkv projection
// [B, (Hq + 2 Hkv) * 128]: the same result as rope_append then
// decode_attention.
void rope_attention(cudaStream_t s, const void* qkv, const float* cos_t, const float* sin_t, const int* pos,
                    void* k_cache, void* v_cache, void* out, int B, int Hq, int Hkv, int Lmax, int splits);
// Sequence splits that give about two CTAs per SM.
int attention_splits(int B, int Hkv, int context, int sms);

// The same two operations on the tensor cores (nab_attn_sm100.cu): per chunk
// of 128 positions, scores K . Q^T and output V^T . P^T as tcgen05 MMAs with
// TMEM accumulators, K/V staged by TMA. splits in [1, 16].
void decode_attention_tc(cudaStream_t s, const void* q, const void* k_cache, const void* v_cache, const int* pos,
                         void* out, int B, int Hq, int Hkv, int Lmax, int splits);
void rope_attention_tc(cudaStream_t s, const void* qkv, const float* cos_t, const float* sin_t, const int* pos,
                       void* k_cache, void* v_cache, void* out, int B, int Hq, int Hkv, int Lmax, int splits);
// Splits for the tensor-core kernel: one CTA per SM, every CTA resident.
int attention_splits_tc(int B, int Hkv, int context, int sms);

// out[B, I] = silu(gu[:, :I]) * gu[:, I:]
void silu_mul(cudaStream_t s, const void* gu, void* out, int B, int I);

}  // namespace nab
