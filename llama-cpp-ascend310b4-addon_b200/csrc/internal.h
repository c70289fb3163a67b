// internal.h -- launchers shared inside libb200_decode.so (not part of the C ABI).
#pragma once

#include <cuda_runtime.h>

#include "args.h"

// GEMV with prologue/epilogue fusion; a.n, a.k, a.w and the fusion fields
// must be set, the tiling fields are filled in from the packed-layout plan.
// pdl: launch with programmatic stream serialisation, so the kernel's
// prologue (weight prefetch) overlaps the tail of the previous kernel in the
// stream; the kernels wait for that kernel before touching its outputs.
int b200i_gemv(int fmt, b200::GemvArgs a, bool debug, cudaStream_t st, bool pdl = false);
int b200i_fa(const b200::FaArgs& a, int head_dim, cudaStream_t st, bool pdl = false);
// CTAs of the tensor-core attention launch for a (one per SM); 0 for head dim 256.
int b200i_fa_ctas(const b200::FaArgs& a, int head_dim);
// Tensor-parallel all-reduce of a.n floats over peer memory (allreduce.cuh).
int b200i_tp_allreduce(const b200::ArArgs& a, cudaStream_t st, bool pdl);
int b200i_sm_count();
int b200i_gemv_grid(int fmt, int64_t n, int64_t k, int epi);
// Sets per-kernel attributes and caches device properties; call before capture.
int b200i_prepare_device();

int b200i_synth_q4_0(uint64_t seed, float sigma, int64_t row0, int64_t nrows, int64_t col0, int64_t ncols,
                     int64_t kglob, void* out, cudaStream_t st);
int b200i_synth_rows_f16(uint64_t seed, uint64_t base, int64_t nrows, int64_t rl, int64_t rg, int64_t col0,
                         void* out, cudaStream_t st);
int b200i_fill_f32(float* p, int64_t n, float v, cudaStream_t st);
int b200i_embed(const void* table, int64_t d_model, int64_t vocab, b200::StepState* state, float* x,
                cudaStream_t st);
int b200i_finish(b200::StepState* state, cudaStream_t st);
// A quantised-activation image (GemvArgs::xq_in layout, U blocks) as ggml
// block_q8_0 rows (U x 34 bytes).
int b200i_image_to_q8_0(const uint8_t* img, int64_t U, uint8_t* out, cudaStream_t st);
