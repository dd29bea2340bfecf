// safetensors_loader.cpp — SafetensorsReader / SafetensorsMultiReader.
//
// Behaviour follows model_loaders/src/safetensors_loader.cpp:29-268 (mmap the
// file, 8-byte little-endian header length, JSON header of {name: {dtype,
// shape, data_offsets}} plus an optional "__metadata__", offsets relative to
// the end of the header; the multi-reader takes the first shard holding a
// name).  The upload goes through pinned staging chunks and the dtype
// conversion runs on the device (hx_convert); the header is validated.
#include "model_loaders/safetensors_loader.h"

#include <cuda_runtime.h>
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <climits>
#include <cstring>
#include <iostream>

#include "hx_kv.h"
#include "json_lite.h"

namespace hxinfer {

namespace {

// Pinned staging chunk: two of them alternate, so the host copy of one chunk
// out of the mapping overlaps the DMA of the other.
constexpr size_t kStageBytes = size_t(16) << 20;

// Bytes per element of the fixed-width safetensors dtypes; 0 = not known here.
size_t dtype_bytes(const std::string& d)
{
    if (d == "F64" || d == "I64" || d == "U64") return 8;
    if (d == "F32" || d == "I32" || d == "U32") return 4;
    if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
    if (d == "I8" || d == "U8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
    return 0;
}

// hx_convert dtype code of a safetensors dtype (0 = not convertible)
int hx_code(const std::string& d)
{
    if (d == "F32") return HX_FP32;
    if (d == "F16") return HX_FP16;
    if (d == "BF16") return HX_BF16;
    return 0;
}

const char* dtype_name(DataType t)
{
    switch (t) {
    case DataType::kDataTypeFP32: return "FP32";
    case DataType::kDataTypeFP16: return "FP16";
    case DataType::kDataTypeInt8: return "Int8";
    default: return "Unknown";
    }
}

void report(const std::string& m)
{
    std::cerr << "[SafetensorsReader] " << m << std::endl;
}

bool cuda_ok(cudaError_t e, const char* what)
{
    if (e == cudaSuccess) return true;
    report(std::string(what) + ": " + cudaGetErrorString(e));
    return false;
}

}  // namespace

SafetensorsReader::~SafetensorsReader()
{
    release_staging();
    unmap();
}

void SafetensorsReader::unmap()
{
    if (mmap_base_) munmap(mmap_base_, file_size_);
    mmap_base_ = nullptr;
    file_size_ = 0;
    tensor_map_.clear();
}

bool SafetensorsReader::load(const std::string& file_path)
{
    unmap();
    path_ = file_path;
    const int fd = open(file_path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        report("Cannot open: " + file_path);
        return false;
    }
    struct stat sb;
    if (fstat(fd, &sb) < 0 || !S_ISREG(sb.st_mode)) {
        close(fd);
        report("not a regular file: " + file_path);
        return false;
    }
    const size_t size = (size_t)sb.st_size;
    if (size < 8) {
        close(fd);
        report(file_path + ": shorter than the 8-byte header length");
        return false;
    }
    void* base = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);  // the mapping keeps the file
    if (base == MAP_FAILED) {
        report("mmap failed: " + file_path);
        return false;
    }
    mmap_base_ = base;
    file_size_ = size;

    const unsigned char* b = static_cast<const unsigned char*>(base);
    uint64_t header_len = 0;
    for (int i = 7; i >= 0; --i) header_len = (header_len << 8) | b[i];  // little-endian
    if (header_len > size - 8) {
        report(file_path + ": header length " + std::to_string(header_len) + " exceeds the file");
        unmap();
        return false;
    }
    const char* h = reinterpret_cast<const char*>(b + 8);
    json_lite::Value root;
    std::string perr;
    if (!json_lite::parse(h, h + header_len, root, &perr)) {
        report(file_path + ": header is not valid JSON: " + perr);
        unmap();
        return false;
    }
    if (root.kind != json_lite::Value::Object) {
        report(file_path + ": header is not a JSON object");
        unmap();
        return false;
    }
    const size_t data_start = 8 + (size_t)header_len;
    const size_t data_size = size - data_start;
    for (const auto& m : root.members) {
        if (m.first == "__metadata__") continue;
        const std::string where = file_path + ": tensor '" + m.first + "': ";
        const json_lite::Value& v = m.second;
        const json_lite::Value* dt = v.find("dtype");
        const json_lite::Value* sh = v.find("shape");
        const json_lite::Value* off = v.find("data_offsets");
        if (!dt || dt->kind != json_lite::Value::String || !sh || sh->kind != json_lite::Value::Array ||
            !off || off->kind != json_lite::Value::Array || off->items.size() != 2) {
            report(where + "needs dtype (string), shape (array) and data_offsets ([begin, end])");
            unmap();
            return false;
        }
        SafetensorInfo info;
        info.dtype = dt->str;
        size_t numel = 1;
        bool too_big = false;
        for (const auto& d : sh->items) {
            if (d.kind != json_lite::Value::Number || !d.is_int || d.integer < 0 || d.integer > INT_MAX) {
                report(where + "shape entries must be integers in [0, INT_MAX]");
                unmap();
                return false;
            }
            info.shape.push_back((int)d.integer);
            if (d.integer && numel > SIZE_MAX / (size_t)d.integer) too_big = true;
            numel *= (size_t)d.integer;
        }
        const json_lite::Value& o0 = off->items[0];
        const json_lite::Value& o1 = off->items[1];
        if (o0.kind != json_lite::Value::Number || !o0.is_int || o1.kind != json_lite::Value::Number ||
            !o1.is_int || o0.integer < 0 || o1.integer < o0.integer || (uint64_t)o1.integer > data_size) {
            report(where + "data_offsets outside the data section of " + std::to_string(data_size) +
                   " bytes");
            unmap();
            return false;
        }
        const size_t nbytes = (size_t)(o1.integer - o0.integer);
        const size_t eb = dtype_bytes(info.dtype);
        if (eb && (too_big || numel > SIZE_MAX / eb || numel * eb != nbytes)) {
            report(where + std::to_string(nbytes) + " bytes do not match its shape and dtype " +
                   info.dtype);
            unmap();
            return false;
        }
        info.offset_begin = data_start + (size_t)o0.integer;
        info.offset_end = data_start + (size_t)o1.integer;
        if (!tensor_map_.emplace(m.first, std::move(info)).second) {
            report(where + "appears twice in the header");
            unmap();
            return false;
        }
    }
    return true;
}

bool SafetensorsReader::has_tensor(const std::string& name) const
{
    return tensor_map_.count(name) > 0;
}

const SafetensorInfo* SafetensorsReader::get_info(const std::string& name) const
{
    auto it = tensor_map_.find(name);
    return it == tensor_map_.end() ? nullptr : &it->second;
}

std::vector<std::string> SafetensorsReader::tensor_names() const
{
    std::vector<std::string> names;
    names.reserve(tensor_map_.size());
    for (const auto& kv : tensor_map_) names.push_back(kv.first);
    std::sort(names.begin(), names.end());
    return names;
}

const void* SafetensorsReader::get_raw_ptr(const std::string& name) const
{
    auto it = tensor_map_.find(name);
    if (it == tensor_map_.end()) return nullptr;
    return static_cast<const char*>(mmap_base_) + it->second.offset_begin;
}

// The reference's dtype-string mapping (safetensors_loader.cpp:100-106).
DataType SafetensorsReader::parse_dtype(const std::string& dtype_str)
{
    if (dtype_str == "F32") return DataType::kDataTypeFP32;
    if (dtype_str == "F16") return DataType::kDataTypeFP16;
    if (dtype_str == "BF16") return DataType::kDataTypeFP16;  // converted on upload
    if (dtype_str == "I8") return DataType::kDataTypeInt8;
    return DataType::kDataTypeFP32;
}

bool SafetensorsReader::ensure_staging() const
{
    int dev = -1;
    if (!cuda_ok(cudaGetDevice(&dev), "cudaGetDevice")) return false;
    if (stream_ && dev == staging_device_) return true;
    release_staging();
    cudaStream_t s = nullptr;
    if (!cuda_ok(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate")) return false;
    stream_ = s;
    staging_device_ = dev;
    for (int i = 0; i < 2; ++i) {
        cudaEvent_t ev = nullptr;
        if (!cuda_ok(cudaHostAlloc(&pinned_[i], kStageBytes, cudaHostAllocDefault), "cudaHostAlloc") ||
            !cuda_ok(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming), "cudaEventCreate")) {
            release_staging();
            return false;
        }
        events_[i] = ev;
    }
    return true;
}

void SafetensorsReader::release_staging() const
{
    if (stream_) cudaStreamSynchronize((cudaStream_t)stream_);
    for (int i = 0; i < 2; ++i) {
        if (events_[i]) cudaEventDestroy((cudaEvent_t)events_[i]);
        if (pinned_[i]) cudaFreeHost(pinned_[i]);
        events_[i] = nullptr;
        pinned_[i] = nullptr;
    }
    if (stream_) cudaStreamDestroy((cudaStream_t)stream_);
    stream_ = nullptr;
    staging_device_ = -1;
}

// Host bytes -> device on stream_, through the two pinned chunks.  Returns
// once every chunk is queued; the caller synchronises the stream.
bool SafetensorsReader::upload(const void* host, void* dev, size_t bytes) const
{
    cudaStream_t s = (cudaStream_t)stream_;
    // start the kernel's read-ahead of the whole range
    const long page = sysconf(_SC_PAGESIZE);
    const uintptr_t h0 = reinterpret_cast<uintptr_t>(host) & ~(uintptr_t)(page - 1);
    madvise(reinterpret_cast<void*>(h0), bytes + (reinterpret_cast<uintptr_t>(host) - h0), MADV_WILLNEED);
    const char* src = static_cast<const char*>(host);
    char* dst = static_cast<char*>(dev);
    int i = 0;
    for (size_t off = 0; off < bytes; off += kStageBytes, i ^= 1) {
        const size_t len = std::min(kStageBytes, bytes - off);
        // the previous DMA out of this chunk has finished (a never-recorded
        // event counts as complete)
        if (!cuda_ok(cudaEventSynchronize((cudaEvent_t)events_[i]), "cudaEventSynchronize")) return false;
        std::memcpy(pinned_[i], src + off, len);
        if (!cuda_ok(cudaMemcpyAsync(dst + off, pinned_[i], len, cudaMemcpyHostToDevice, s),
                     "cudaMemcpyAsync"))
            return false;
        if (!cuda_ok(cudaEventRecord((cudaEvent_t)events_[i], s), "cudaEventRecord")) return false;
    }
    return true;
}

std::shared_ptr<Tensor> SafetensorsReader::get_tensor_gpu(const std::string& name,
                                                          const std::shared_ptr<CUDAAllocator>& alloc,
                                                          DataType target_dtype) const
{
    auto it = tensor_map_.find(name);
    if (it == tensor_map_.end()) {
        report("Tensor not found: " + name);
        return nullptr;
    }
    if (!alloc) {
        report("null allocator for " + name);
        return nullptr;
    }
    const SafetensorInfo& info = it->second;
    const int src = hx_code(info.dtype);
    const int dst = target_dtype == DataType::kDataTypeFP32   ? HX_FP32
                    : target_dtype == DataType::kDataTypeFP16 ? HX_FP16
                                                              : 0;
    const bool int8_copy = info.dtype == "I8" && target_dtype == DataType::kDataTypeInt8;
    if (!int8_copy && (!src || !dst)) {
        report("unsupported conversion " + info.dtype + " -> " + dtype_name(target_dtype) + " for " +
               name);
        return nullptr;
    }
    size_t n = 1;
    for (int d : info.shape) n *= (size_t)d;  // bounded when the header was read
    const size_t raw = info.offset_end - info.offset_begin;

    auto t = std::make_shared<Tensor>(alloc, info.shape, target_dtype);
    t->tensor_set_device_type(DeviceType::kDeviceCUDA);
    if (n == 0) return t;
    if (!t->raw_data_ptr()) {
        report("device allocation of " + std::to_string(t->tensor_total_byte_size()) +
               " bytes failed for " + name);
        return nullptr;
    }
    if (!ensure_staging()) return nullptr;
    cudaStream_t s = (cudaStream_t)stream_;
    const char* host = static_cast<const char*>(mmap_base_) + info.offset_begin;

    // Same element size: the raw bytes land in the tensor (converted in place
    // for BF16 -> FP16).  Otherwise they land in a temporary and are converted
    // into the tensor.
    void* landing = t->raw_data_ptr();
    void* temp = nullptr;
    if (raw != t->tensor_total_byte_size()) {
        if (!cuda_ok(cudaMallocAsync(&temp, raw, s), "cudaMallocAsync")) return nullptr;
        landing = temp;
    }
    bool ok = upload(host, landing, raw);
    if (ok && !int8_copy && src != dst) {
        const int rc = hx_convert(t->raw_data_ptr(), dst, landing, src, n, s);
        if (rc != HX_OK) {
            report(std::string("hx_convert: ") + hx_last_error());
            ok = false;
        }
    }
    if (temp) ok = cuda_ok(cudaFreeAsync(temp, s), "cudaFreeAsync") && ok;
    ok = cuda_ok(cudaStreamSynchronize(s), "cudaStreamSynchronize") && ok;
    return ok ? t : nullptr;
}

// ------------------------------------------------------------ multi-shard reader

bool SafetensorsMultiReader::load_directory(const std::string& dir_path)
{
    readers_.clear();
    tensor_to_shard_.clear();
    std::vector<std::string> files;
    if (DIR* d = opendir(dir_path.c_str())) {
        const std::string ext = ".safetensors";
        while (const dirent* e = readdir(d)) {
            const std::string n = e->d_name;
            // what the shell glob dir/*.safetensors matches: no hidden names
            if (n.size() > ext.size() && n[0] != '.' &&
                n.compare(n.size() - ext.size(), ext.size(), ext) == 0)
                files.push_back(dir_path + "/" + n);
        }
        closedir(d);
    }
    std::sort(files.begin(), files.end());
    if (files.empty()) files.push_back(dir_path + "/model.safetensors");
    for (const auto& f : files) {
        auto r = std::make_unique<SafetensorsReader>();
        if (!r->load(f)) continue;
        const int idx = (int)readers_.size();
        for (const auto& name : r->tensor_names()) tensor_to_shard_.emplace(name, idx);
        readers_.push_back(std::move(r));
    }
    return !readers_.empty();
}

bool SafetensorsMultiReader::has_tensor(const std::string& name) const
{
    return tensor_to_shard_.count(name) > 0;
}

std::shared_ptr<Tensor> SafetensorsMultiReader::get_tensor_gpu(const std::string& name,
                                                               const std::shared_ptr<CUDAAllocator>& alloc,
                                                               DataType target_dtype) const
{
    auto it = tensor_to_shard_.find(name);
    if (it == tensor_to_shard_.end()) {
        std::cerr << "[SafetensorsMultiReader] Tensor not found: " << name << std::endl;
        return nullptr;
    }
    return readers_[it->second]->get_tensor_gpu(name, alloc, target_dtype);
}

size_t SafetensorsMultiReader::num_tensors() const
{
    size_t total = 0;
    for (const auto& r : readers_) total += r->num_tensors();
    return total;
}

std::vector<std::string> SafetensorsMultiReader::tensor_names() const
{
    std::vector<std::string> names;
    names.reserve(tensor_to_shard_.size());
    for (const auto& kv : tensor_to_shard_) names.push_back(kv.first);
    std::sort(names.begin(), names.end());
    return names;
}

}  // namespace hxinfer
