/*
 * sa_attention_cuda.h -- C++ host API of the CUDA method for the streaming
 * attention functions of the reference's attention/src/attention.h.
 *
 * Each function takes the same arguments, with the same meaning, as the
 * reference function it stands beside: host row-major fp32 buffers
 * (Q [d], K and V [T x d]), no 1/sqrt(d) scale, the result returned by value
 * as a std::vector<float> of d elements owned by the caller.  A driver that
 * selects a method by name adds "cuda" next to "serial" / "omp" / "mpi" and
 * calls these.  Implemented in libsa_host.so over the C ABI of libsa_cuda.so
 * (include/sa_cuda.h); the device work is the single-pass split-KV decode
 * kernel, so the naive and streaming variants give the same result up to fp32
 * rounding, as the reference's own variants do.
 *
 * Errors: attention.h has no error returns (bad sizes are undefined
 * behaviour there).  These functions throw std::invalid_argument for sizes
 * the GPU path does not support (d outside {64, 128, 256}, T < 0,
 * block_size <= 0, num_gpus outside 1..available) and std::runtime_error for
 * CUDA failures, with the library's message.  T = 0 returns zeros, as the
 * reference's serial code does.
 *
 * Threading: process-wide state is one sa_ctx per GPU, created on first use
 * and guarded by a mutex per GPU, so calls from several host threads are
 * serialised per device.
 */
#ifndef SA_ATTENTION_CUDA_H
#define SA_ATTENTION_CUDA_H

#include <vector>

/* naive_attention_serial / naive_attention_omp (attention.h:27-55). */
std::vector<float> naive_attention_cuda(const float* Q, const float* K, const float* V, int T, int d);

/* streaming_attention_serial / streaming_attention_omp (attention.h:123-129,
 * 157-165).  block_size is the reference's online-softmax block; it must be
 * positive and does not change the result beyond fp32 rounding. */
std::vector<float> streaming_attention_cuda(const float* Q, const float* K, const float* V, int T, int d,
                                            int block_size);

/* streaming_attention_mpi_simple (attention.h:199-208) inside one process:
 * the T keys are split into num_gpus contiguous slices (the reference's
 * rank partition), GPU i computes the online-softmax state (m, l, O) of its
 * slice, and the states are merged (merge_partial_results,
 * streaming_omp.cpp:27-48).  The result is the full output (the reference
 * returns it on rank 0 only). */
std::vector<float> streaming_attention_cuda_multi(const float* Q, const float* K, const float* V, int T, int d,
                                                  int block_size, int num_gpus);

/* GPU used by naive_attention_cuda / streaming_attention_cuda (default 0). */
void attention_cuda_set_device(int device);
/* Number of GPUs visible to this process. */
int attention_cuda_device_count();
/* Destroy the per-GPU contexts (they are otherwise released at exit). */
void attention_cuda_release();

#endif /* SA_ATTENTION_CUDA_H */
