// rows.h — [rows, cols] activation buffers that grow on demand, for the
// n-row TransformerLayer, SwigluLayer and CausalLMModel of this directory.
#ifndef HXINFER_B200_ENGINE_ROWS_H
#define HXINFER_B200_ENGINE_ROWS_H
#include <algorithm>
#include <memory>
#include <vector>

#include "tensor/tensor.h"

namespace hxinfer {

// Rows to allocate for n: the next power of two, at most max_rows (and at
// least n).
inline int grown_rows(int n, int max_rows)
{
    int cap = 1;
    while (cap < n) cap *= 2;
    return std::max(n, std::min(cap, max_rows));
}

// (Re)allocates t as [cap, cols] on `allocator`'s device.
inline void alloc_rows(const std::shared_ptr<Allocator>& allocator, std::shared_ptr<Tensor>& t, int cap,
                       int cols, DataType dtype)
{
    t = std::make_shared<Tensor>(allocator, std::vector<int>{cap, cols}, dtype);
    t->tensor_set_device_type(allocator->device_type());
}

}  // namespace hxinfer
#endif
