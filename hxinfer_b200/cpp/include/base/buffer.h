// base/buffer.h — one allocation owned through an Allocator
// (interface of hxinfer-engine/include/base/buffer.h:7-18), or a non-owning
// view of memory owned elsewhere.
#ifndef HXINFER_B200_BUFFER_H
#define HXINFER_B200_BUFFER_H
#include <cstddef>
#include <memory>

#include "base/allocator.h"

namespace hxinfer {

class Buffer {
public:
    Buffer(std::shared_ptr<Allocator> allocator, size_t byte_size);
    Buffer(void* external, size_t byte_size);  // view; never released
    ~Buffer();
    Buffer(const Buffer&) = delete;
    Buffer& operator=(const Buffer&) = delete;
    size_t buffer_byte_size() const { return byte_size_; }
    const void* buffer_data_ptr() const { return data_; }
    void* buffer_data_ptr() { return data_; }

private:
    std::shared_ptr<Allocator> allocator_;
    size_t byte_size_ = 0;
    void* data_ = nullptr;
};

}  // namespace hxinfer
#endif
