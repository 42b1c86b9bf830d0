// Decode-step kernels of the tensor-parallel Llama model (nab_llama.cu).
#pragma once

#include <cuda_runtime.h>

namespace nab {

// Rotary embedding of q and k (head_dim 128, half-split convention) and append
// of k, v at position *pos of the caches [B, Hkv, Lmax, 128].
void rope_append(cudaStream_t s, const void* qkv, const float* cos_t, const float* sin_t, const int* pos,
                 void* q_out, void* k_cache, void* v_cache, int B, int Hq, int Hkv, int Lmax);

// GQA decode attention over positions [0, *pos]; part_ml holds B*Hq*splits*2
// floats and part_o B*Hq*splits*128 floats of scratch; counters B*Hkv ints
// that start at zero (the kernel leaves them at zero).
void decode_attention(cudaStream_t s, const void* q, const void* k_cache, const void* v_cache, const int* pos,
                      float* part_ml, float* part_o, int* counters, void* out, int B, int Hq, int Hkv, int Lmax,
                      int splits);
// Sequence splits that give about two CTAs per SM.
int attention_splits(int B, int Hkv, int context, int sms);

// out[B, I] = silu(gu[:, :I]) * gu[:, I:]
void silu_mul(cudaStream_t s, const void* gu, void* out, int B, int I);

}  // namespace nab
