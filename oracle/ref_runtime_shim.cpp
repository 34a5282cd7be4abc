// Host-memory CUDA runtime used when the reference world generator is built in
// its CUDA CPU-fallback mode (reference: src/gpu/cuda/cpu_fallback/
// CudaRuntimeCpuFallback.h:154-226 declares these entry points; the
// reference's own definitions live in CudaRuntimeCpuFallback.cpp, which needs
// a Vulkan stack and is therefore not compiled here). Streams and events are
// no-ops because the fallback launcher runs every kernel synchronously.
//
// Test infrastructure only: this shim exists so the oracle can run the
// reference's own code. It is never linked into the product library.

#include <gpu/cuda/cpu_fallback/CudaRuntimeCpuFallback.h>

#include <cstdlib>
#include <cstring>

thread_local dim3 threadIdx;
thread_local dim3 blockIdx;
thread_local dim3 blockDim;
thread_local dim3 gridDim;

const char* cudaGetErrorString(cudaError_t error)
{
    return error == cudaSuccess ? "no error" : "host shim error";
}

cudaError_t cudaMallocHost(void** ptr, std::size_t size)
{
    *ptr = std::malloc(size ? size : 1);
    return *ptr ? cudaSuccess : cudaErrorMemoryAllocation;
}

cudaError_t cudaFreeHost(void* ptr)
{
    std::free(ptr);
    return cudaSuccess;
}

cudaError_t cudaMalloc(void** ptr, std::size_t size) { return cudaMallocHost(ptr, size); }
cudaError_t cudaFree(void* ptr) { return cudaFreeHost(ptr); }

cudaError_t cudaMemcpy(void* dst, const void* src, std::size_t count, cudaMemcpyKind)
{
    if (count)
        std::memmove(dst, src, count);
    return cudaSuccess;
}

cudaError_t cudaMemcpyAsync(void* dst, const void* src, std::size_t count, cudaMemcpyKind kind, cudaStream_t)
{
    return cudaMemcpy(dst, src, count, kind);
}

cudaError_t cudaMemsetAsync(void* ptr, int value, std::size_t count, cudaStream_t)
{
    std::memset(ptr, value, count);
    return cudaSuccess;
}

cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned)
{
    static int token;
    *e = &token;
    return cudaSuccess;
}
cudaError_t cudaEventDestroy(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaEventRecord(cudaEvent_t, cudaStream_t) { return cudaSuccess; }
cudaError_t cudaEventSynchronize(cudaEvent_t) { return cudaSuccess; }
cudaError_t cudaEventQuery(cudaEvent_t) { return cudaSuccess; }

cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned)
{
    static int token;
    *s = &token;
    return cudaSuccess;
}
cudaError_t cudaStreamDestroy(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaStreamWaitEvent(cudaStream_t, cudaEvent_t, unsigned) { return cudaSuccess; }
