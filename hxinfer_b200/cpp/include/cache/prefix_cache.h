// cache/prefix_cache.h — PrefixCacheManager with the reference's interface
// (hxinfer-engine/include/cache/prefix_cache.h:16-155): construct from an
// allocator and a ModelConfig; store / lookup / restore a token prefix;
// cache_size.  The hash is the same FNV-1a 64 (prefix_cache.h:42-49) and the
// semantics are the same: store snapshots the first prefix_len positions of
// every layer's K and V; lookup returns prefix_len on an exact token match and
// 0 on a miss or a hash collision; restore finds the snapshot by hash and
// copies it back into the first prefix_len positions, leaving later positions
// untouched; a restore miss prints an error and returns.
//
// What changes: the copies are device kernels (hx_kv_snapshot /
// hx_kv_restore) on the legacy default stream, ordered with the model's own
// launches, and each layer's K and V snapshot is one buffer from `allocator`.
// With a device allocator (CUDAAllocator, DeviceAllocator) snapshots stay in
// device memory.  With a CPUAllocator (what the reference's callers pass: its
// snapshots are host tensors) they stay in host memory, as in the reference,
// and move through a device staging buffer with a synchronous cudaMemcpy.
// store/restore accept any model type whose get_blocks()[i]->get_attention()
// yields this build's AttentionLayer (LlamaModel, Qwen2Model, CausalLMModel).
#ifndef HXINFER_B200_PREFIX_CACHE_H
#define HXINFER_B200_PREFIX_CACHE_H
#include <cuda_runtime.h>

#include <cstdint>
#include <iostream>
#include <memory>
#include <unordered_map>
#include <vector>

#include "base/allocator.h"
#include "base/config.h"
#include "hx_kv.h"
#include "layer/attention.h"
#include "tensor/tensor.h"

namespace hxinfer {

class PrefixCacheManager {
private:
    struct CachedKVBlock {
        std::vector<int> token_ids;
        int prefix_len;
        std::vector<std::shared_ptr<Tensor>> layer_kv;  // per layer: K and V snapshot
    };
    std::unordered_map<size_t, std::shared_ptr<CachedKVBlock>> cache_map_;
    std::shared_ptr<Allocator> allocator_;
    ModelConfig config_;
    std::shared_ptr<Tensor> staging_;  // device copy of one layer's snapshot (host snapshots)

    bool host_snapshots() const
    {
        return allocator_ && allocator_->device_type() == DeviceType::kDeviceCPU;
    }
    // Device buffer of at least `bytes` bytes for host-resident snapshots.
    void* staging(size_t bytes)
    {
        if (!staging_ || staging_->tensor_total_byte_size() < bytes)
            staging_ = std::make_shared<Tensor>(std::make_shared<CUDAAllocator>(),
                                                std::vector<int>{static_cast<int>(bytes)},
                                                DataType::kDataTypeInt8);
        return staging_->raw_data_ptr();
    }

    size_t compute_hash(const std::vector<int>& tokens) const
    {
        return (size_t)hx_prefix_hash(reinterpret_cast<const int32_t*>(tokens.data()), tokens.size());
    }

public:
    PrefixCacheManager(std::shared_ptr<Allocator> allocator, ModelConfig config)
        : allocator_(allocator), config_(config) {}

    template <class Model>
    void store(const std::vector<int>& prefix_tokens, Model& model)
    {
        const size_t hash = compute_hash(prefix_tokens);
        const int prefix_len = static_cast<int>(prefix_tokens.size());
        auto block = std::make_shared<CachedKVBlock>();
        block->token_ids = prefix_tokens;
        block->prefix_len = prefix_len;
        auto& blocks = model.get_blocks();
        for (int i = 0; i < config_.layer; i++) {
            hx_kv_cache* kv = blocks[i]->get_attention()->kv_cache();
            const size_t bytes = hx_snapshot_bytes(kv, prefix_len);
            auto snap = std::make_shared<Tensor>(
                allocator_, std::vector<int>{static_cast<int>(bytes > 0 ? bytes : 1)},
                DataType::kDataTypeInt8);
            if (!snap->raw_data_ptr()) {
                std::cerr << "[PrefixCache] store failed: snapshot allocation of " << bytes
                          << " bytes" << std::endl;
                return;
            }
            int rc;
            if (host_snapshots() && bytes > 0) {
                void* dev = staging(bytes);
                rc = dev ? hx_kv_snapshot(kv, 0, prefix_len, dev, bytes, nullptr) : HX_ERR_OOM;
                if (rc == HX_OK &&
                    cudaMemcpy(snap->raw_data_ptr(), dev, bytes, cudaMemcpyDeviceToHost) != cudaSuccess)
                    rc = HX_ERR_CUDA;
            } else {
                rc = hx_kv_snapshot(kv, 0, prefix_len, snap->raw_data_ptr(), bytes, nullptr);
            }
            if (rc != HX_OK) {
                std::cerr << "[PrefixCache] store failed: " << hx_status_string(rc) << " ("
                          << hx_last_error() << ")" << std::endl;
                return;
            }
            block->layer_kv.push_back(snap);
        }
        cache_map_[hash] = block;
        std::cout << "[PrefixCache] stored prefix (" << prefix_len << " tokens, " << config_.layer
                  << " layers, hash=" << hash << ")" << std::endl;
    }

    int lookup(const std::vector<int>& prefix_tokens) const
    {
        auto it = cache_map_.find(compute_hash(prefix_tokens));
        if (it == cache_map_.end()) return 0;
        return it->second->token_ids == prefix_tokens ? it->second->prefix_len : 0;
    }

    template <class Model>
    void restore(const std::vector<int>& prefix_tokens, Model& model)
    {
        auto it = cache_map_.find(compute_hash(prefix_tokens));
        if (it == cache_map_.end()) {
            std::cerr << "[PrefixCache] restore failed: prefix not cached" << std::endl;
            return;
        }
        const auto& block = it->second;
        auto& blocks = model.get_blocks();
        for (int i = 0; i < config_.layer; i++) {
            hx_kv_cache* kv = blocks[i]->get_attention()->kv_cache();
            const auto& snap = block->layer_kv[i];
            const size_t bytes = hx_snapshot_bytes(kv, block->prefix_len);
            int rc;
            if (host_snapshots() && bytes > 0) {
                void* dev = staging(bytes);
                rc = dev ? HX_OK : HX_ERR_OOM;
                if (rc == HX_OK &&
                    cudaMemcpy(dev, snap->raw_data_ptr(), bytes, cudaMemcpyHostToDevice) != cudaSuccess)
                    rc = HX_ERR_CUDA;
                if (rc == HX_OK) rc = hx_kv_restore(kv, 0, block->prefix_len, dev, bytes, nullptr);
            } else {
                rc = hx_kv_restore(kv, 0, block->prefix_len, snap->raw_data_ptr(),
                                   snap->tensor_total_byte_size(), nullptr);
            }
            if (rc != HX_OK) {
                std::cerr << "[PrefixCache] restore failed: " << hx_status_string(rc) << " ("
                          << hx_last_error() << ")" << std::endl;
                return;
            }
        }
        std::cout << "[PrefixCache] restored prefix (" << block->prefix_len << " tokens)"
                  << std::endl;
    }

    size_t cache_size() const { return cache_map_.size(); }
};

}  // namespace hxinfer
#endif
