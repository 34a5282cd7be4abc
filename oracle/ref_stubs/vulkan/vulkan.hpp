// Empty Vulkan handle types: the reference's CUDA CPU-fallback runtime header
// names vk::Device / vk::DeviceMemory / vk::Semaphore in interop structs that
// the world generator never touches (reference:
// src/gpu/cuda/cpu_fallback/CudaRuntimeCpuFallback.h:117-176).
//
// Test infrastructure only; never linked into the product library.
#pragma once

namespace vk {
struct Device {};
struct DeviceMemory {};
struct Semaphore {};
} // namespace vk
