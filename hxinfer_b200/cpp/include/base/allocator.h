// base/allocator.h — the Allocator interface of the reference
// (hxinfer-engine/include/base/allocator.h:7-27) and its CPU/CUDA
// allocators, plus DeviceAllocator: stream-ordered allocations from a CUDA
// memory pool that keeps freed memory for reuse, every size rounded up to a
// multiple of 128 bytes.  The KV cache and snapshots of this build come from
// it.  Allocation failures return nullptr (as CUDAAllocator::allocate does in
// the reference, allocator_cuda.cu:11-17).
#ifndef HXINFER_B200_ALLOCATOR_H
#define HXINFER_B200_ALLOCATOR_H
#include <cstddef>

#include "base/config.h"

namespace hxinfer {

class Allocator {
public:
    virtual void* allocate(size_t byte_size) = 0;
    virtual void release(void* ptr) = 0;
    virtual ~Allocator() = default;
    virtual DeviceType device_type() = 0;
};

class CPUAllocator : public Allocator {
public:
    void* allocate(size_t byte_size) override;
    void release(void* ptr) override;
    DeviceType device_type() override { return DeviceType::kDeviceCPU; }
};

class CUDAAllocator : public Allocator {
public:
    void* allocate(size_t byte_size) override;
    void release(void* ptr) override;
    DeviceType device_type() override { return DeviceType::kDeviceCUDA; }
};

class DeviceAllocator : public Allocator {
public:
    static constexpr size_t kAlign = 128;
    void* allocate(size_t byte_size) override;
    void release(void* ptr) override;
    DeviceType device_type() override { return DeviceType::kDeviceCUDA; }
};

}  // namespace hxinfer
#endif
