// model_loaders/safetensors_loader.h — safetensors checkpoint reader with the
// reference's interface (model_loaders/include/safetensors_loader.h:17-67):
// SafetensorInfo, SafetensorsReader (one file) and SafetensorsMultiReader (a
// directory of shards), same member names, argument meaning and failure
// behaviour (a message on stderr, then false / nullptr).
//
// What changes underneath:
//  - upload: the file is mmap'd and its raw bytes go to the device through two
//    pinned staging chunks (host copy of chunk i+1 overlapping the DMA of
//    chunk i) instead of a pageable cudaMemcpy;
//  - dtype conversion (BF16 -> FP16 / FP32, FP32 -> FP16, FP16 -> FP32) runs
//    on the device (hx_convert in libhxkv.so), in place for BF16 -> FP16,
//    instead of a CPU loop per element (safetensors_loader.cpp:12-27, 124-197);
//  - the header is validated (header length, data offsets inside the file,
//    byte size = elements x dtype size) and a pair the reference would copy
//    byte-for-byte into a tensor of another dtype (its fallback,
//    safetensors_loader.cpp:200-205) is refused instead;
//  - tensor_names() lists the tensors (the reference's returns an empty list).
#ifndef HXINFER_B200_SAFETENSORS_LOADER_H
#define HXINFER_B200_SAFETENSORS_LOADER_H
#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "tensor/tensor.h"

namespace hxinfer {

struct SafetensorInfo {
    std::string dtype;         // safetensors dtype string: "F32", "F16", "BF16", "I8", ...
    std::vector<int> shape;
    size_t offset_begin;       // byte offsets from the start of the file
    size_t offset_end;
};

class SafetensorsReader {
public:
    SafetensorsReader() = default;
    ~SafetensorsReader();
    SafetensorsReader(const SafetensorsReader&) = delete;
    SafetensorsReader& operator=(const SafetensorsReader&) = delete;

    // Maps the file and parses its header; false (message on stderr) if the
    // file cannot be opened or the header is malformed.
    bool load(const std::string& file_path);
    bool has_tensor(const std::string& name) const;
    const SafetensorInfo* get_info(const std::string& name) const;
    size_t num_tensors() const { return tensor_map_.size(); }
    std::vector<std::string> tensor_names() const;

    // Host pointer to the tensor's bytes inside the mapping (nullptr if absent).
    const void* get_raw_ptr(const std::string& name) const;

    // A new CUDA tensor of `target_dtype` holding the named tensor, converted
    // on the device.  Pairs: F32/F16/BF16 -> FP16 or FP32, I8 -> Int8.
    // nullptr (message on stderr) if the tensor is absent, the pair is not
    // supported, or an allocation or CUDA call fails.  Synchronous: the data
    // is in place when the call returns.  One reader serves one thread at a
    // time (its staging buffers are shared between calls), as the reference's
    // reader does.
    std::shared_ptr<Tensor> get_tensor_gpu(const std::string& name,
                                           const std::shared_ptr<CUDAAllocator>& alloc,
                                           DataType target_dtype = DataType::kDataTypeFP16) const;

private:
    static DataType parse_dtype(const std::string& dtype_str);
    void unmap();
    bool upload(const void* host, void* dev, size_t bytes) const;
    bool ensure_staging() const;
    void release_staging() const;

    void* mmap_base_ = nullptr;
    size_t file_size_ = 0;
    std::string path_;
    std::unordered_map<std::string, SafetensorInfo> tensor_map_;

    // Created on the first get_tensor_gpu, on the device current then.
    mutable int staging_device_ = -1;
    mutable void* stream_ = nullptr;  // cudaStream_t
    mutable void* pinned_[2] = {nullptr, nullptr};
    mutable void* events_[2] = {nullptr, nullptr};  // cudaEvent_t
};

class SafetensorsMultiReader {
public:
    // Reads every *.safetensors file of the directory (sorted by name), or
    // model.safetensors when there is none; true if at least one file loaded.
    bool load_directory(const std::string& dir_path);
    bool has_tensor(const std::string& name) const;
    std::shared_ptr<Tensor> get_tensor_gpu(const std::string& name,
                                           const std::shared_ptr<CUDAAllocator>& alloc,
                                           DataType target_dtype = DataType::kDataTypeFP16) const;
    size_t num_tensors() const;
    std::vector<std::string> tensor_names() const;

private:
    std::vector<std::unique_ptr<SafetensorsReader>> readers_;
    std::unordered_map<std::string, int> tensor_to_shard_;  // first shard holding each name
};

}  // namespace hxinfer
#endif
