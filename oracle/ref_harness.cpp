// C entry points around the reference's own world generator and observation
// conversion, so the oracle can run the UNMODIFIED reference code
// (reference: src/world/WorldGenerator.cu:673-829 `WorldGenerator::Impl::generate`,
// reached through the raw overload declared at src/world/WorldGenerator.h:82,
// and src/environment/CudaObservation.cu:34-44 `convertRgba8ToFloatNchw`).
//
// The same file is compiled twice by oracle/Makefile:
//   * with g++ against the reference's CUDA CPU-fallback launcher
//     (CUDA_CPU_FALLBACK_MODE) -> oracle/_ref/libref_cpu.so, the CPU baseline;
//   * with nvcc for sm_100a against the real CUDA runtime
//     -> oracle/_ref/libref_cuda.so, the reference CUDA path.
// Test infrastructure only: nothing in the product links or loads it.

#include <world/Block.h>
#include <world/Voxel.h>
#include <blocklab/gpu/cuda/CudaFuture.h>
#include <blocklab/utility/Math.h>
#include <environment/Agent.h>
#include <gpu/cuda/PageLockedVector.h>
#include <environment/CudaObservation.h>

#include <cuda_runtime.h>

#include <chrono>
#include <cstdint>
#include <cstring>
#include <memory>
#include <span>
#include <utility>
#include <vector>

// The raw generate(WorldGenerationInput, ...) overload is private in the
// reference; opening it here lets the oracle drive the generator on explicit
// regions and override lists, exactly as the reference's tests do through
// World (tests/WorldTestUtils.cpp:135-170).
#define private public
#include <world/WorldGenerator.h>
#undef private

namespace {

struct DeviceBuffer {
    void* ptr = nullptr;
    explicit DeviceBuffer(std::size_t bytes) { cudaMalloc(&ptr, bytes ? bytes : 1); }
    ~DeviceBuffer() { cudaFree(ptr); }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};

} // namespace

extern "C" {

// Runs `runs` consecutive generations of the same region with one generator
// (runs >= 2 reaches the converged light-source capacity, see
// src/world/WorldGenerator.cu:705-711) and copies out the last one.
//   overrides: n_overrides * (x, y, z) int32 world coordinates + block ids
//   out_block/out_block_light/out_sky_light: W*H*D bytes, index x + W*(y + H*z)
//   out_height_map: W*D int8, index x + W*z
//   out_voxels: max_voxels * 12 bytes (may be null when max_voxels == 0)
//   out_run_ms: wall time of each generation including its readback, `runs`
//               entries (may be null)
// Returns 0 on success.
int ref_generate(std::uint32_t seed, std::int32_t origin_x, std::int32_t origin_y, std::int32_t origin_z,
    std::uint32_t width, std::uint32_t height, std::uint32_t depth,
    const std::int32_t* override_xyz, const std::uint8_t* override_block, std::uint32_t n_overrides,
    std::int32_t runs,
    std::uint8_t* out_block, std::uint8_t* out_block_light, std::uint8_t* out_sky_light,
    std::int8_t* out_height_map,
    void* out_voxels, std::uint32_t max_voxels, std::uint32_t* out_voxel_count, std::int32_t* out_header,
    double* out_run_ms)
{
    using namespace blocklab;
    std::vector<BlockOverride> overrides(n_overrides);
    for (std::uint32_t i = 0; i < n_overrides; ++i) {
        overrides[i].coord = IVec3 { override_xyz[3 * i], override_xyz[3 * i + 1], override_xyz[3 * i + 2] };
        overrides[i].block = static_cast<Block>(override_block[i]);
    }

    const std::size_t volume = static_cast<std::size_t>(width) * height * depth;
    DeviceBuffer header(sizeof(TerrainHeader));
    DeviceBuffer voxels(static_cast<std::size_t>(VoxelSize) * (max_voxels ? max_voxels : 1));

    WorldGenerator generator;
    WorldGenerationInput input;
    input.seed = seed;
    input.worldVersion = 1;
    input.center = IVec3 { origin_x + static_cast<std::int32_t>(width / 2), origin_y,
        origin_z + static_cast<std::int32_t>(depth / 2) };
    input.size = UVec3 { width, height, depth };
    input.origin = IVec3 { origin_x, origin_y, origin_z };
    input.overrides = std::span<const BlockOverride>(overrides.data(), overrides.size());

    CPUCacheGenerationBuffers cache;
    std::uint32_t voxel_count = 0;
    for (std::int32_t r = 0; r < (runs < 1 ? 1 : runs); ++r) {
        const auto t0 = std::chrono::steady_clock::now();
        WorldGenerationBuffers buffers {
            .terrain = {
                .header = static_cast<TerrainHeader*>(header.ptr),
                .voxels = static_cast<Voxel*>(voxels.ptr),
                .maxVoxels = max_voxels,
            },
            .cpuCache = std::move(cache),
        };
        auto future = generator.generate(input, std::move(buffers));
        WorldGenerationOutput& out = future.get();
        voxel_count = out.voxelCount;
        cache = std::move(out.buffers.cpuCache);
        if (out_run_ms)
            out_run_ms[r] = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    }

    for (std::size_t i = 0; i < volume; ++i) {
        out_block[i] = static_cast<std::uint8_t>(cache.blocks[i].blockType);
        out_block_light[i] = static_cast<std::uint8_t>(cache.blocks[i].blockLight);
        out_sky_light[i] = static_cast<std::uint8_t>(cache.blocks[i].skyLight);
    }
    for (std::size_t i = 0; i < static_cast<std::size_t>(width) * depth; ++i)
        out_height_map[i] = cache.heightMap[i];
    if (out_voxel_count)
        *out_voxel_count = voxel_count;
    if (out_voxels && max_voxels)
        cudaMemcpy(out_voxels, voxels.ptr, static_cast<std::size_t>(VoxelSize) * voxel_count, cudaMemcpyDeviceToHost);
    if (out_header)
        cudaMemcpy(out_header, header.ptr, sizeof(TerrainHeader), cudaMemcpyDeviceToHost);
#ifdef CUDA_CPU_FALLBACK_MODE
    return 0;
#else
    return static_cast<int>(cudaDeviceSynchronize());
#endif
}

#ifndef CUDA_CPU_FALLBACK_MODE
// Device time of the reference's own kernels for one generation, without its
// host work (override packing and sort) and its copies (override upload,
// block-cache readback): `runs` generations converge the light-source
// capacity, the next generation is captured from the generator's stream into
// a CUDA graph, and a graph of only its kernel and memset nodes, in captured
// order, is launched `reps` times between CUDA events. *out_kernel_ms gets the
// mean time per generation and *out_wall_ms the wall time of one ordinary
// generation (kernels, copies and host work). Returns 0 on success.
int ref_kernel_time(std::uint32_t seed, std::int32_t origin_x, std::int32_t origin_y, std::int32_t origin_z,
    std::uint32_t width, std::uint32_t height, std::uint32_t depth, const std::int32_t* override_xyz,
    const std::uint8_t* override_block, std::uint32_t n_overrides, std::int32_t runs, std::int32_t reps,
    double* out_kernel_ms, double* out_wall_ms)
{
    using namespace blocklab;
    std::vector<BlockOverride> overrides(n_overrides);
    for (std::uint32_t i = 0; i < n_overrides; ++i) {
        overrides[i].coord = IVec3 { override_xyz[3 * i], override_xyz[3 * i + 1], override_xyz[3 * i + 2] };
        overrides[i].block = static_cast<Block>(override_block[i]);
    }
    DeviceBuffer header(sizeof(TerrainHeader));
    DeviceBuffer voxels(VoxelSize);
    WorldGenerator generator;
    WorldGenerationInput input;
    input.seed = seed;
    input.worldVersion = 1;
    input.center = IVec3 { origin_x + static_cast<std::int32_t>(width / 2), origin_y,
        origin_z + static_cast<std::int32_t>(depth / 2) };
    input.size = UVec3 { width, height, depth };
    input.origin = IVec3 { origin_x, origin_y, origin_z };
    input.overrides = std::span<const BlockOverride>(overrides.data(), overrides.size());
    CPUCacheGenerationBuffers cache;
    auto one = [&]() {
        WorldGenerationBuffers buffers {
            .terrain = { .header = static_cast<TerrainHeader*>(header.ptr), .voxels = static_cast<Voxel*>(voxels.ptr),
                .maxVoxels = 0 },
            .cpuCache = std::move(cache),
        };
        return generator.generate(input, std::move(buffers));
    };
    for (std::int32_t r = 0; r < (runs < 1 ? 1 : runs); ++r) {
        const auto t0 = std::chrono::steady_clock::now();
        auto f = one();
        cache = std::move(f.get().buffers.cpuCache);
        if (out_wall_ms)
            *out_wall_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    }
    cudaStream_t st = generator.stream();
    cudaGraph_t captured = nullptr;
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed) != cudaSuccess)
        return 1;
    auto pending = one();
    if (cudaStreamEndCapture(st, &captured) != cudaSuccess || !captured)
        return 2;
    // The captured generation is a chain: walk it from its root.
    std::size_t n = 0;
    cudaGraphGetNodes(captured, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    cudaGraphGetNodes(captured, nodes.data(), &n);
    cudaGraphNode_t cur = nullptr;
    for (cudaGraphNode_t node : nodes) {
        std::size_t deps = 0;
        cudaGraphNodeGetDependencies(node, nullptr, &deps);
        if (deps == 0)
            cur = node;
    }
    cudaGraph_t kernels = nullptr;
    cudaGraphCreate(&kernels, 0);
    cudaGraphNode_t last = nullptr;
    std::size_t kept = 0;
    while (cur) {
        cudaGraphNodeType type;
        cudaGraphNodeGetType(cur, &type);
        cudaGraphNode_t added = nullptr;
        if (type == cudaGraphNodeTypeKernel) {
            cudaKernelNodeParams p {};
            cudaGraphKernelNodeGetParams(cur, &p);
            cudaGraphAddKernelNode(&added, kernels, last ? &last : nullptr, last ? 1 : 0, &p);
        } else if (type == cudaGraphNodeTypeMemset) {
            cudaMemsetParams p {};
            cudaGraphMemsetNodeGetParams(cur, &p);
            cudaGraphAddMemsetNode(&added, kernels, last ? &last : nullptr, last ? 1 : 0, &p);
        }
        if (added) {
            last = added;
            ++kept;
        }
        std::size_t next = 0;
        cudaGraphNodeGetDependentNodes(cur, nullptr, &next);
        if (next == 0)
            break;
        std::vector<cudaGraphNode_t> after(next);
        cudaGraphNodeGetDependentNodes(cur, after.data(), &next);
        cur = after[0];
    }
    cudaGraphExec_t exec = nullptr;
    if (kept == 0 || cudaGraphInstantiate(&exec, kernels, 0) != cudaSuccess)
        return 3;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaGraphLaunch(exec, st); // warm-up
    cudaEventRecord(e0, st);
    for (std::int32_t r = 0; r < (reps < 1 ? 1 : reps); ++r)
        cudaGraphLaunch(exec, st);
    cudaEventRecord(e1, st);
    cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (out_kernel_ms)
        *out_kernel_ms = ms / (reps < 1 ? 1 : reps);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    cudaGraphDestroy(kernels);
    cudaGraphDestroy(captured);
    return static_cast<int>(cudaDeviceSynchronize());
}
#endif

// Reference RGBA8 -> float32 NCHW conversion on host buffers
// (src/environment/CudaObservation.cu:34-44); `rgba` is batch*height*width*4
// bytes, `nchw` batch*3*height*width floats.
int ref_convert_rgba8(const std::uint8_t* rgba, float* nchw, std::uint32_t batch, std::uint32_t width,
    std::uint32_t height)
{
    const std::size_t pixels = static_cast<std::size_t>(batch) * width * height;
    DeviceBuffer in(pixels * 4);
    DeviceBuffer out(pixels * 3 * sizeof(float));
    cudaMemcpy(in.ptr, rgba, pixels * 4, cudaMemcpyHostToDevice);
    blocklab::convertRgba8ToFloatNchw(in.ptr, static_cast<float*>(out.ptr), batch, width, height, 0);
    cudaMemcpy(nchw, out.ptr, pixels * 3 * sizeof(float), cudaMemcpyDeviceToHost);
#ifdef CUDA_CPU_FALLBACK_MODE
    return 0;
#else
    return static_cast<int>(cudaDeviceSynchronize());
#endif
}

} // extern "C"
