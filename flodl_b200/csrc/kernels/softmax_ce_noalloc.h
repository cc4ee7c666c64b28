// C interface of the allocation-free softmax cross-entropy
// (softmax_ce_noalloc.cu).
//
// This interface has no counterpart in the reference (fab2s/floDl); it is an
// addition of this library for callers that cannot allocate device memory
// where they need the loss: a serving runtime that owns a fixed memory pool,
// or a plug-in that may only use the buffers it is handed. These callers pass
// their inputs and outputs; the scratch lives in a fixed device array of the
// library (about 1 MiB per GPU that loads it, held until the process exits).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

// Return codes besides 0 (success) and positive cudaError_t values.
#define FLODL_NOALLOC_ERR_TOO_MANY_ROWS (-1)  // T above flodl_softmax_ce_noalloc_max_rows()
#define FLODL_NOALLOC_ERR_BAD_ARGS (-2)       // non-positive sizes, ld < V, null pointers

#ifdef __cplusplus
extern "C" {
#endif

// Fused softmax cross-entropy that allocates nothing.
//   logits   : bf16 [T, V], row pitch `ld` elements (device)
//   targets  : int64 [T] (device); rows equal to ignore_index are skipped.
//              A target outside [0, V) that is not ignore_index is never used
//              as an index: the row is skipped like an ignored one and counted
//              in the bad-row count that flodl_softmax_ce_noalloc_bad_rows reads.
//   loss_out : f32 scalar (device), receives the mean loss over the valid rows
//   dlogits  : bf16 [T, V] contiguous (device) or NULL, receives d(mean loss)/dlogits
//   stream   : CUDA stream to launch on (0 = legacy default stream)
// The first call on a device looks up the scratch array's device address and
// caches it; make that first call before any stream capture. Calls that
// overlap on the GPU share the scratch array and race; serialise them on one
// stream.
int flodl_softmax_ce_noalloc(const void* logits, int ld, const int64_t* targets, int T, int V,
                             int64_t ignore_index, float smoothing, float* loss_out, void* dlogits,
                             cudaStream_t stream);

// Capacity of the fixed scratch array, in rows.
int flodl_softmax_ce_noalloc_max_rows(void);

// Number of rows of the last call on the current device whose target was
// outside [0, V) and not ignore_index. Waits for `stream` (the stream of that
// call), then copies one word into *out. Returns 0 or a positive cudaError_t.
int flodl_softmax_ce_noalloc_bad_rows(cudaStream_t stream, int* out);

#ifdef __cplusplus
}
#endif
