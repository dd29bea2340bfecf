// base.cpp — allocators, Buffer and Tensor of the C++ interface layer.
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <iostream>
#include <new>
#include <numeric>
#include <stdexcept>

#include "base/allocator.h"
#include "base/buffer.h"
#include "tensor/tensor.h"

namespace hxinfer {

void* CPUAllocator::allocate(size_t byte_size)
{
    void* p = nullptr;
    if (posix_memalign(&p, 64, byte_size ? byte_size : 64) != 0 || !p) throw std::bad_alloc();
    std::memset(p, 0, byte_size);
    return p;
}

void CPUAllocator::release(void* p) { std::free(p); }

void* CUDAAllocator::allocate(size_t byte_size)
{
    if (byte_size == 0) return nullptr;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, byte_size);
    if (e != cudaSuccess) {
        std::cerr << "[hxinfer] cudaMalloc of " << byte_size << " bytes failed: "
                  << cudaGetErrorString(e) << std::endl;
        return nullptr;
    }
    return p;
}

void CUDAAllocator::release(void* p)
{
    if (p) cudaFree(p);
}

void* DeviceAllocator::allocate(size_t byte_size)
{
    if (byte_size == 0) return nullptr;
    const size_t bytes = (byte_size + kAlign - 1) / kAlign * kAlign;
    static bool pool_ready[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !pool_ready[dev]) {
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
            uint64_t keep = UINT64_MAX;  // keep freed memory in the pool for reuse
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        }
        pool_ready[dev] = true;
    }
    void* p = nullptr;
    cudaError_t e = cudaMallocAsync(&p, bytes, nullptr);
    if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
    if (e != cudaSuccess) {
        std::cerr << "[hxinfer] device allocation of " << bytes << " bytes failed: "
                  << cudaGetErrorString(e) << std::endl;
        return nullptr;
    }
    return p;
}

void DeviceAllocator::release(void* p)
{
    if (p) cudaFreeAsync(p, nullptr);
}

Buffer::Buffer(std::shared_ptr<Allocator> allocator, size_t byte_size)
    : allocator_(std::move(allocator)), byte_size_(byte_size)
{
    data_ = allocator_->allocate(byte_size_);
}

Buffer::Buffer(void* external, size_t byte_size) : byte_size_(byte_size), data_(external) {}

Buffer::~Buffer()
{
    if (data_ && allocator_) allocator_->release(data_);
    data_ = nullptr;
}

static size_t product(const std::vector<int>& s)
{
    return std::accumulate(s.begin(), s.end(), size_t{1},
                           [](size_t a, int b) { return a * static_cast<size_t>(b); });
}

Tensor::Tensor(std::shared_ptr<Allocator> allocator, std::vector<int> shapes, DataType data_type)
    : shapes_(std::move(shapes)), data_type_(data_type)
{
    total_elements_ = product(shapes_);
    total_byte_size_ = total_elements_ * DataTypeSize(data_type_);
    buffer_ = std::make_shared<Buffer>(allocator, total_byte_size_);
    device_type_ = allocator->device_type();
}

Tensor::Tensor(void* data, std::vector<int> shapes, DataType data_type, DeviceType device)
    : shapes_(std::move(shapes)), data_type_(data_type), device_type_(device)
{
    total_elements_ = product(shapes_);
    total_byte_size_ = total_elements_ * DataTypeSize(data_type_);
    buffer_ = std::make_shared<Buffer>(data, total_byte_size_);
}

void Tensor::tensor_reshape(std::vector<int> new_shapes)
{
    const size_t n = product(new_shapes);
    if (n * DataTypeSize(data_type_) > total_byte_size_)
        throw std::runtime_error("tensor_reshape: new shape does not fit the allocation");
    total_elements_ = n;
    shapes_ = std::move(new_shapes);
}

std::shared_ptr<Tensor> Tensor::tensor_to_cuda(std::shared_ptr<CUDAAllocator> cuda_allocator)
{
    if (device_type_ == DeviceType::kDeviceCUDA) return std::make_shared<Tensor>(*this);
    auto t = std::make_shared<Tensor>(cuda_allocator, shapes_, data_type_);
    cudaError_t e = cudaMemcpy(t->raw_data_ptr(), raw_data_ptr(), total_byte_size_,
                               cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        std::cerr << "[hxinfer] tensor_to_cuda failed: " << cudaGetErrorString(e) << std::endl;
        return nullptr;
    }
    t->tensor_set_device_type(DeviceType::kDeviceCUDA);
    return t;
}

std::shared_ptr<Tensor> Tensor::tensor_to_cpu(std::shared_ptr<CPUAllocator> cpu_allocator)
{
    if (device_type_ == DeviceType::kDeviceCPU) return std::make_shared<Tensor>(*this);
    auto t = std::make_shared<Tensor>(cpu_allocator, shapes_, data_type_);
    cudaError_t e = cudaMemcpy(t->raw_data_ptr(), raw_data_ptr(), total_byte_size_,
                               cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        std::cerr << "[hxinfer] tensor_to_cpu failed: " << cudaGetErrorString(e) << std::endl;
        return nullptr;
    }
    t->tensor_set_device_type(DeviceType::kDeviceCPU);
    return t;
}

}  // namespace hxinfer
