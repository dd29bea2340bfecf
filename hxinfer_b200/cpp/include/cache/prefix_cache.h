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
// What changes: the copies are device kernels on the legacy default stream,
// ordered with the model's own launches: one hx_kv_snapshot_layers /
// hx_kv_restore_layers launch covers every layer (up to 64 per launch), and a
// prefix's K and V of all layers is one buffer from `allocator`.  With a
// device allocator (CUDAAllocator, DeviceAllocator) snapshots stay in device
// memory.  With a CPUAllocator (what the reference's callers pass: its
// snapshots are host tensors) they stay in host memory, as in the reference,
// and move through one device staging buffer with one synchronous
// cudaMemcpy per store or restore.
// store/restore accept any model type whose get_blocks()[i]->get_attention()
// yields this build's AttentionLayer (LlamaModel, Qwen2Model, CausalLMModel).
#ifndef HXINFER_B200_PREFIX_CACHE_H
#define HXINFER_B200_PREFIX_CACHE_H
#include <cuda_runtime.h>

#include <algorithm>
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
        // every layer's K and V snapshot, one buffer [layer][K|V][kv_head][prefix_len][head_dim]
        std::shared_ptr<Tensor> kv;
        size_t layer_bytes;
    };
    std::unordered_map<size_t, std::shared_ptr<CachedKVBlock>> cache_map_;
    std::shared_ptr<Allocator> allocator_;
    ModelConfig config_;
    std::shared_ptr<Tensor> staging_;  // device copy of a whole snapshot (host snapshots)

    bool host_snapshots() const
    {
        return allocator_ && allocator_->device_type() == DeviceType::kDeviceCPU;
    }
    // Device buffer of at least `bytes` bytes for host-resident snapshots.
    void* staging(size_t layers, size_t layer_bytes)
    {
        const size_t bytes = layers * layer_bytes;
        if (!staging_ || staging_->tensor_total_byte_size() < bytes)
            staging_ = std::make_shared<Tensor>(
                std::make_shared<CUDAAllocator>(),
                std::vector<int>{static_cast<int>(layers), static_cast<int>(layer_bytes)},
                DataType::kDataTypeInt8);
        return staging_->raw_data_ptr();
    }

    size_t compute_hash(const std::vector<int>& tokens) const
    {
        return (size_t)hx_prefix_hash(reinterpret_cast<const int32_t*>(tokens.data()), tokens.size());
    }

    // Copies positions [0, prefix_len) of every layer's cache into (to_snapshot)
    // or out of `buf` (device memory, layer i at i * layer_bytes): one launch
    // per 64 layers when the layers hold one-layer wrapped caches (this
    // build's AttentionLayer), else one launch per layer.
    template <class Model>
    int copy_layers(Model& model, int prefix_len, char* buf, size_t layer_bytes, bool to_snapshot)
    {
        auto& blocks = model.get_blocks();
        std::vector<hx_kv_cache*> caches(config_.layer);
        for (int i = 0; i < config_.layer; i++) caches[i] = blocks[i]->get_attention()->kv_cache();
        for (int i0 = 0; i0 < config_.layer; i0 += 64) {
            const int n = std::min(64, config_.layer - i0);
            char* at = buf + (size_t)i0 * layer_bytes;
            int rc = to_snapshot
                ? hx_kv_snapshot_layers(caches.data() + i0, n, prefix_len, at, n * layer_bytes, nullptr)
                : hx_kv_restore_layers(caches.data() + i0, n, prefix_len, at, n * layer_bytes, nullptr);
            if (rc == HX_ERR_INVALID) {  // not all one-layer wrapped caches: layer by layer
                rc = HX_OK;
                for (int i = 0; i < n && rc == HX_OK; i++)
                    rc = to_snapshot
                        ? hx_kv_snapshot(caches[i0 + i], 0, prefix_len, at + i * layer_bytes, layer_bytes, nullptr)
                        : hx_kv_restore(caches[i0 + i], 0, prefix_len, at + i * layer_bytes, layer_bytes, nullptr);
            }
            if (rc != HX_OK) return rc;
        }
        return HX_OK;
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
        hx_kv_cache* kv0 = model.get_blocks()[0]->get_attention()->kv_cache();
        block->layer_bytes = hx_snapshot_bytes(kv0, prefix_len);
        const size_t layer_bytes = block->layer_bytes > 0 ? block->layer_bytes : 16;
        block->kv = std::make_shared<Tensor>(
            allocator_, std::vector<int>{config_.layer, static_cast<int>(layer_bytes)},
            DataType::kDataTypeInt8);
        if (!block->kv->raw_data_ptr()) {
            std::cerr << "[PrefixCache] store failed: snapshot allocation of "
                      << config_.layer * layer_bytes << " bytes" << std::endl;
            return;
        }
        int rc = HX_OK;
        if (prefix_len > 0) {
            if (host_snapshots()) {
                void* dev = staging(config_.layer, block->layer_bytes);
                rc = dev ? copy_layers(model, prefix_len, static_cast<char*>(dev), block->layer_bytes, true)
                         : HX_ERR_OOM;
                if (rc == HX_OK && cudaMemcpy(block->kv->raw_data_ptr(), dev,
                                              config_.layer * block->layer_bytes,
                                              cudaMemcpyDeviceToHost) != cudaSuccess)
                    rc = HX_ERR_CUDA;
            } else {
                rc = copy_layers(model, prefix_len, static_cast<char*>(block->kv->raw_data_ptr()),
                                 block->layer_bytes, true);
            }
        }
        if (rc != HX_OK) {
            std::cerr << "[PrefixCache] store failed: " << hx_status_string(rc) << " ("
                      << hx_last_error() << ")" << std::endl;
            return;
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
        int rc = HX_OK;
        if (block->prefix_len > 0) {
            if (host_snapshots()) {
                void* dev = staging(config_.layer, block->layer_bytes);
                rc = dev ? HX_OK : HX_ERR_OOM;
                if (rc == HX_OK && cudaMemcpy(dev, block->kv->raw_data_ptr(),
                                              config_.layer * block->layer_bytes,
                                              cudaMemcpyHostToDevice) != cudaSuccess)
                    rc = HX_ERR_CUDA;
                if (rc == HX_OK)
                    rc = copy_layers(model, block->prefix_len, static_cast<char*>(dev), block->layer_bytes, false);
            } else {
                rc = copy_layers(model, block->prefix_len, static_cast<char*>(block->kv->raw_data_ptr()),
                                 block->layer_bytes, false);
            }
        }
        if (rc != HX_OK) {
            std::cerr << "[PrefixCache] restore failed: " << hx_status_string(rc) << " ("
                      << hx_last_error() << ")" << std::endl;
            return;
        }
        std::cout << "[PrefixCache] restored prefix (" << block->prefix_len << " tokens)"
                  << std::endl;
    }

    size_t cache_size() const { return cache_map_.size(); }
};

}  // namespace hxinfer
#endif
