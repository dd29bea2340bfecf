// tensor/tensor.h — shape, dtype, device tag and a shared Buffer.
// Same member functions as hxinfer-engine/include/tensor/tensor.h:13-64 so
// callers of the reference Tensor compile unchanged.
#ifndef HXINFER_B200_TENSOR_H
#define HXINFER_B200_TENSOR_H
#include <cstddef>
#include <memory>
#include <vector>

#include "base/allocator.h"
#include "base/buffer.h"
#include "base/config.h"

namespace hxinfer {

class Tensor {
public:
    Tensor(std::shared_ptr<Allocator> allocator, std::vector<int> shapes, DataType data_type);
    // Non-owning view of existing memory on `device`.
    Tensor(void* data, std::vector<int> shapes, DataType data_type, DeviceType device);
    ~Tensor() = default;

    const std::vector<int>& tensor_shapes() const { return shapes_; }
    DataType tensor_data_type() const { return data_type_; }
    size_t tensor_total_elements() const { return total_elements_; }
    size_t tensor_total_byte_size() const { return total_byte_size_; }
    DeviceType tensor_device_type() const { return device_type_; }
    void tensor_set_device_type(DeviceType t) { device_type_ = t; }
    // Changes the shape within the allocation; throws if it would not fit.
    void tensor_reshape(std::vector<int> new_shapes);

    template <typename T>
    const T* tensor_data_ptr() const { return static_cast<const T*>(buffer_->buffer_data_ptr()); }
    template <typename T>
    T* tensor_data_ptr() { return static_cast<T*>(buffer_->buffer_data_ptr()); }
    const void* raw_data_ptr() const { return buffer_->buffer_data_ptr(); }
    void* raw_data_ptr() { return buffer_->buffer_data_ptr(); }

    std::shared_ptr<Tensor> tensor_to_cuda(std::shared_ptr<CUDAAllocator> cuda_allocator);
    std::shared_ptr<Tensor> tensor_to_cpu(std::shared_ptr<CPUAllocator> cpu_allocator);

private:
    std::vector<int> shapes_;
    DataType data_type_;
    size_t total_elements_ = 0;
    size_t total_byte_size_ = 0;
    std::shared_ptr<Buffer> buffer_;
    DeviceType device_type_ = DeviceType::kDeviceCPU;
};

}  // namespace hxinfer
#endif
