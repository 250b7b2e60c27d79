// Host-only stand-in for the CUDA runtime declarations the C API uses, so
// csrc/runtime/capi.cc builds and runs with g++ on a machine without a GPU.
// "Device" memory is host memory and every stream completes immediately,
// except that a test can hold all events not-ready to model a hung stream.
#pragma once
#include <stddef.h>
#include <stdint.h>

enum cudaError { cudaSuccess = 0, cudaErrorInvalidValue = 1, cudaErrorNotReady = 600 };
typedef enum cudaError cudaError_t;
enum cudaMemcpyKind { cudaMemcpyHostToHost = 0, cudaMemcpyHostToDevice = 1, cudaMemcpyDeviceToHost = 2,
                      cudaMemcpyDeviceToDevice = 3, cudaMemcpyDefault = 4 };
typedef struct CUstream_st* cudaStream_t;
typedef struct CUevent_st* cudaEvent_t;
#define cudaEventDisableTiming 2
#define cudaStreamNonBlocking 1

cudaError_t cudaMalloc(void** p, size_t bytes);
template <typename T>
inline cudaError_t cudaMalloc(T** p, size_t bytes) { return cudaMalloc(reinterpret_cast<void**>(p), bytes); }
cudaError_t cudaFree(void* p);
cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind);
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes, cudaMemcpyKind kind, cudaStream_t s = 0);
cudaError_t cudaMemsetAsync(void* dst, int value, size_t bytes, cudaStream_t s = 0);
cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned int flags);
cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t s = 0);
cudaError_t cudaEventQuery(cudaEvent_t e);
cudaError_t cudaEventDestroy(cudaEvent_t e);
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned int flags);
cudaError_t cudaStreamDestroy(cudaStream_t s);
cudaError_t cudaStreamSynchronize(cudaStream_t s);
cudaError_t cudaDeviceSynchronize();
const char* cudaGetErrorString(cudaError_t e);

// test controls
namespace vb_stub {
void set_streams_hung(bool hung);        // events stay not-ready while set
int interp_launches();                   // launch_interp calls so far
}
