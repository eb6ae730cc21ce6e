// hx_container.h — reader of Hearth's `.hearth` container (version 1) for the MoE path: the preamble,
// the metadata keys the path uses, the tensor and expert directories, all validated against the
// format's rules (docs/FORMAT.md §1-§6 of the reference; the reference reads the same file in
// engine/src/modelfile.c), and positioned reads of tensors and expert slabs. Host code only.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace hx {

struct CtTensor {
    std::string name;
    uint32_t dtype = 0, ndim = 0;
    uint32_t shape[4] = {1, 1, 1, 1};   // outermost first
    uint64_t off = 0, nbytes = 0;
};

struct CtExpert {
    uint64_t off = 0, nbytes = 0;   // nbytes 0: no slab (a dense layer)
    uint32_t dtype = 0, flags = 0;  // flags bit 0: aliased (shares its slab with another entry)
};

struct Container {
    uint64_t file_bytes = 0;
    // metadata keys of the MoE path, defaults applied (FORMAT §3.1)
    uint32_t n_layers = 0, d_model = 0, vocab_size = 0, n_heads = 0;
    uint32_t n_experts = 0, top_k = 0, expert_ffn_dim = 0, shared_ffn_dim = 0, shared_gate = 0;
    uint32_t score_fn = 0, score_bias = 0, n_group = 1, topk_group = 1, norm_topk_prob = 0;
    float norm_eps = 1e-6f, routed_scale = 1.0f, residual_scale = 1.0f;
    // the rest of the decoder (FORMAT §3.1 keys, defaults applied as engine/src/modelfile.c does)
    uint32_t max_seq = 4096, attn_kind = 0, n_kv_heads = 0, head_dim = 0, qk_norm = 0, qkv_bias = 0;
    uint32_t rope_dim = 0, rope_style = 0, dense_ffn_dim = 0, tie_embeddings = 0;
    float rope_attn_factor = 1.0f, attn_scale = 1.0f, emb_scale = 1.0f, logit_scale = 1.0f;
    std::vector<uint8_t> layer_kind;   // per layer: 0 dense FFN, 1 MoE
    std::vector<CtTensor> tensors;
    std::unordered_map<std::string, size_t> by_name;
    std::vector<CtExpert> experts;     // [n_layers * n_experts], index layer * n_experts + e
    int n_moe_layers = 0, n_physical = 0, n_aliased = 0;
    int expert_dtype = -1;             // dtype shared by every slab; -1 when mixed or none

    const CtTensor *find(const std::string &name) const {
        auto it = by_name.find(name);
        return it == by_name.end() ? nullptr : &tensors[it->second];
    }
};

// An open container file: parse() validates everything before any data is used.
class ContainerFile {
public:
    ContainerFile() = default;
    ~ContainerFile();
    ContainerFile(const ContainerFile &) = delete;
    ContainerFile &operator=(const ContainerFile &) = delete;

    // false with a message for an unreadable file or any violation of the format
    bool open(const char *path, std::string &err);
    const Container &info() const { return c_; }
    // n bytes at absolute offset off into dst
    bool read(uint64_t off, void *dst, size_t n, std::string &err) const;

private:
    bool parse(std::string &err);
    int fd_ = -1;
    Container c_;
};

}  // namespace hx
