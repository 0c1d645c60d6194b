// C declarations of the allocation-free AdamW entry point (noalloc_adamw.cu).
//
// This interface has no counterpart in the reference implementation.  It is for
// callers of this library that cannot allocate device memory; the rules of use
// (one static device table of at most 1024 tensors per call, calls serialised on
// the GPU, no call during stream capture) are stated beside the definitions.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Status codes returned by tfb_adamw_multi_noalloc.
enum {
  TFB_NOALLOC_OK = 0,
  TFB_NOALLOC_TOO_MANY_TENSORS = 1,  // n_tensors > tfb_adamw_noalloc_max_tensors(); nothing launched
  TFB_NOALLOC_BAD_ARGUMENT = 2,      // null pointer, empty tensor, n_tensors < 1 or too many elements
  TFB_NOALLOC_CUDA_ERROR = 3,        // a CUDA call failed; the message names it
};

// Largest number of tensors one call accepts (the size of the static device table).
int tfb_adamw_noalloc_max_tensors(void);

// Message of the calling thread's last failed call (empty after a success).
const char* tfb_adamw_noalloc_last_error(void);

// One AdamW step over n_tensors fp32 tensors, in place, on `stream`, with no device
// allocation.  params / grads / exp_avgs / exp_avg_sqs: host arrays of device pointers;
// numels, bias1 (1 - beta1^step), bias2 (1 - beta2^step): host arrays, one entry per
// tensor; lr_dev: device pointer to the fp32 learning rate.
int tfb_adamw_multi_noalloc(float* const* params, const float* const* grads, float* const* exp_avgs,
                            float* const* exp_avg_sqs, const long long* numels, const float* bias1,
                            const float* bias2, int n_tensors, const float* lr_dev, double beta1, double beta2,
                            float eps, float weight_decay, int cautious, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
