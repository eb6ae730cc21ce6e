// hx_container.cpp — `.hearth` container reader for the MoE path (see hx_container.h).
#include "hx_container.h"

#include <cmath>

#include <algorithm>
#include <cerrno>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

namespace hx {

namespace {

constexpr uint32_t kMagic = 0x48545248u;   // "HRTH"
constexpr uint32_t kVersion = 1u;
constexpr uint64_t kSlabAlign = 4096u, kTensorAlign = 64u;
constexpr size_t kPreamble = 64, kTensorEntry = 128, kExpertEntry = 32, kNameLen = 80;
constexpr uint32_t kFlagAliased = 1u;

// the format is little-endian, like every host this library builds for
uint16_t rd16(const uint8_t *p) { uint16_t v; std::memcpy(&v, p, 2); return v; }
uint32_t rd32(const uint8_t *p) { uint32_t v; std::memcpy(&v, p, 4); return v; }
uint64_t rd64(const uint8_t *p) { uint64_t v; std::memcpy(&v, p, 8); return v; }

uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

// FORMAT §6 row bytes; 0 for an unknown dtype or a block dtype whose row is not whole blocks
uint64_t row_bytes_of(uint32_t dtype, uint64_t n) {
    switch (dtype) {
    case 0: return 4 * n;                         // F32
    case 1: case 2: return 2 * n;                 // F16, BF16
    case 3: return n % 64 ? 0 : n / 64 * 66;      // Q8
    case 4: return n % 64 ? 0 : n / 64 * 34;      // Q4
    case 5: return 4 * n;                         // I32
    case 6: return n;                             // U8
    default: return 0;
    }
}

// FORMAT §5 slab size of an expert of dtype with gate/up [F, D] and down [D, F]; 0 if impossible
uint64_t slab_size(uint32_t dtype, uint64_t D, uint64_t F) {
    const uint64_t rd = row_bytes_of(dtype, D), rf = row_bytes_of(dtype, F);
    if (!rd || !rf) return 0;
    const uint64_t up = align_up(F * rd, 64), down = align_up(up + F * rd, 64);
    return align_up(down + D * rf, kSlabAlign);
}

struct MetaVal {
    uint8_t type = 0;
    uint64_t u = 0;        // types 1, 3
    float f = 0.0f;        // type 2
    std::vector<uint8_t> bytes;   // type 7 (and the raw payload of 4, 5, 6)
};

std::string fmt(const char *f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char *f, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, f);
    vsnprintf(buf, sizeof buf, f, ap);
    va_end(ap);
    return buf;
}

}  // namespace

ContainerFile::~ContainerFile() {
    if (fd_ >= 0) ::close(fd_);
}

bool ContainerFile::read(uint64_t off, void *dst, size_t n, std::string &err) const {
    if (off > c_.file_bytes || n > c_.file_bytes - off) {
        err = fmt("read of %zu bytes at %llu is past the end of the file", n, (unsigned long long)off);
        return false;
    }
    uint8_t *p = static_cast<uint8_t *>(dst);
    while (n) {
        const ssize_t r = ::pread(fd_, p, n, (off_t)off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) {
            err = fmt("read at %llu failed: %s", (unsigned long long)off, r < 0 ? std::strerror(errno) : "end of file");
            return false;
        }
        p += r;
        off += (uint64_t)r;
        n -= (size_t)r;
    }
    return true;
}

bool ContainerFile::open(const char *path, std::string &err) {
    if (fd_ >= 0) ::close(fd_);
    c_ = Container();
    fd_ = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) {
        err = fmt("cannot open %s: %s", path, std::strerror(errno));
        return false;
    }
    struct stat st;
    if (fstat(fd_, &st) != 0) {
        err = fmt("cannot stat %s: %s", path, std::strerror(errno));
        return false;
    }
    c_.file_bytes = (uint64_t)st.st_size;
    return parse(err);
}

bool ContainerFile::parse(std::string &err) {
    Container &c = c_;
    const uint64_t fsz = c.file_bytes;
    auto inside = [&](uint64_t off, uint64_t n) { return off <= fsz && n <= fsz - off; };

    // ---- §2 preamble
    uint8_t pre[kPreamble];
    if (fsz < kPreamble) {
        err = "file shorter than the 64-byte preamble";
        return false;
    }
    if (!read(0, pre, kPreamble, err)) return false;
    if (rd32(pre) != kMagic) {
        err = fmt("bad magic 0x%08x (expected 0x%08x)", rd32(pre), kMagic);
        return false;
    }
    if (rd32(pre + 4) != kVersion) {
        err = fmt("unsupported version %u", rd32(pre + 4));
        return false;
    }
    const uint64_t meta_off = rd64(pre + 8), meta_bytes = rd64(pre + 16), tdir_off = rd64(pre + 24),
                   n_tensors = rd64(pre + 32), edir_off = rd64(pre + 40), n_entries = rd64(pre + 48);
    if (rd32(pre + 56) != kSlabAlign) {
        err = fmt("slab alignment %u (must be 4096)", rd32(pre + 56));
        return false;
    }
    if (n_tensors > fsz / kTensorEntry || n_entries > fsz / kExpertEntry || !inside(meta_off, meta_bytes) ||
        !inside(tdir_off, n_tensors * kTensorEntry) || !inside(edir_off, n_entries * kExpertEntry)) {
        err = "metadata or a directory lies outside the file";
        return false;
    }

    // ---- §3 metadata
    std::vector<uint8_t> mb(meta_bytes);
    if (meta_bytes && !read(meta_off, mb.data(), mb.size(), err)) return false;
    std::unordered_map<std::string, MetaVal> meta;
    for (size_t pos = 0; pos < mb.size();) {
        auto need = [&](size_t n) { return n <= mb.size() - pos; };
        if (!need(2)) {
            err = "truncated metadata entry";
            return false;
        }
        const size_t klen = rd16(&mb[pos]);
        pos += 2;
        if (!need(klen + 1)) {
            err = "truncated metadata entry";
            return false;
        }
        std::string key(reinterpret_cast<const char *>(&mb[pos]), klen);
        pos += klen;
        MetaVal v;
        v.type = mb[pos++];
        size_t payload;
        switch (v.type) {
        case 1: case 2: payload = 4; break;
        case 3: payload = 8; break;
        case 4: case 5: case 6: case 7: {
            if (!need(4)) {
                err = fmt("truncated metadata value of %s", key.c_str());
                return false;
            }
            const uint64_t cnt = rd32(&mb[pos]);
            pos += 4;
            payload = (size_t)(v.type == 4 || v.type == 7 ? cnt : cnt * 4);
            break;
        }
        default:
            err = fmt("metadata key %s has unknown type %u", key.c_str(), v.type);
            return false;
        }
        if (!need(payload)) {
            err = fmt("truncated metadata value of %s", key.c_str());
            return false;
        }
        if (v.type == 1) v.u = rd32(&mb[pos]);
        else if (v.type == 3) v.u = rd64(&mb[pos]);
        else if (v.type == 2) std::memcpy(&v.f, &mb[pos], 4);
        else v.bytes.assign(mb.begin() + (ptrdiff_t)pos, mb.begin() + (ptrdiff_t)(pos + payload));
        pos += payload;
        if (!meta.emplace(key, std::move(v)).second) {
            err = fmt("metadata key %s appears twice", key.c_str());
            return false;
        }
    }
    auto get_u32 = [&](const char *k, uint32_t def, bool required, uint32_t &out) {
        auto it = meta.find(k);
        if (it == meta.end()) {
            if (required) err = fmt("metadata is missing required key %s", k);
            out = def;
            return !required;
        }
        if ((it->second.type != 1 && it->second.type != 3) || it->second.u > 0xffffffffull) {
            err = fmt("metadata %s must be a u32", k);
            return false;
        }
        out = (uint32_t)it->second.u;
        return true;
    };
    auto get_f32 = [&](const char *k, float def, float &out) {
        auto it = meta.find(k);
        if (it == meta.end()) {
            out = def;
            return true;
        }
        if (it->second.type != 2) {
            err = fmt("metadata %s must be an f32", k);
            return false;
        }
        out = it->second.f;
        return true;
    };
    if (!get_u32("n_layers", 0, true, c.n_layers) || !get_u32("d_model", 0, true, c.d_model) ||
        !get_u32("vocab_size", 0, true, c.vocab_size) || !get_u32("n_heads", 0, true, c.n_heads) ||
        !get_u32("n_experts", 0, false, c.n_experts) || !get_u32("top_k", 0, false, c.top_k) ||
        !get_u32("expert_ffn_dim", 0, false, c.expert_ffn_dim) ||
        !get_u32("shared_ffn_dim", 0, false, c.shared_ffn_dim) || !get_u32("shared_gate", 0, false, c.shared_gate) ||
        !get_u32("score_fn", 0, false, c.score_fn) || !get_u32("score_bias", 0, false, c.score_bias) ||
        !get_u32("n_group", 1, false, c.n_group) || !get_u32("topk_group", 1, false, c.topk_group) ||
        !get_u32("norm_topk_prob", 0, false, c.norm_topk_prob) || !get_f32("norm_eps", 1e-6f, c.norm_eps) ||
        !get_f32("routed_scale", 1.0f, c.routed_scale) || !get_f32("residual_scale", 1.0f, c.residual_scale))
        return false;
    if (!c.n_layers || !c.d_model || !c.vocab_size || !c.n_heads) {
        err = "n_layers, d_model, vocab_size and n_heads must be positive";
        return false;
    }
    // attention and dense keys (engine/src/modelfile.c:235-290): GQA / MHA only here; an MLA
    // container keeps attn_kind 1 and is refused by the whole-model handle, not by the reader
    {
        uint32_t qk_rope = 0;
        if (!get_u32("max_seq", 4096, false, c.max_seq) || !get_u32("attn_kind", 0, false, c.attn_kind) ||
            !get_u32("n_kv_heads", c.n_heads, false, c.n_kv_heads) ||
            !get_u32("head_dim", c.d_model / c.n_heads, false, c.head_dim) ||
            !get_u32("qk_norm", 0, false, c.qk_norm) || !get_u32("qkv_bias", 0, false, c.qkv_bias) ||
            !get_u32("qk_rope_dim", 0, false, qk_rope) || !get_u32("rope_style", 0, false, c.rope_style) ||
            !get_u32("dense_ffn_dim", 0, false, c.dense_ffn_dim) ||
            !get_u32("tie_embeddings", 0, false, c.tie_embeddings) ||
            !get_f32("rope_attn_factor", 1.0f, c.rope_attn_factor) || !get_f32("emb_scale", 1.0f, c.emb_scale) ||
            !get_f32("logit_scale", 1.0f, c.logit_scale))
            return false;
        const uint32_t rope_cap = c.attn_kind == 1 ? qk_rope : c.head_dim;
        if (!get_u32("rope_dim", rope_cap, false, c.rope_dim)) return false;
        if (c.attn_kind == 0) {
            if (!c.head_dim || !c.n_kv_heads || c.n_heads % c.n_kv_heads || c.qk_norm > 2 || c.rope_dim > c.head_dim ||
                c.rope_dim % 2 || c.rope_style > 1) {
                err = "attention keys out of range (head_dim, n_kv_heads, qk_norm, rope_dim, rope_style)";
                return false;
            }
            // float arithmetic, as hearth.format.apply_defaults and modelfile.c compute it
            if (!get_f32("attn_scale", 1.0f / sqrtf((float)c.head_dim), c.attn_scale)) return false;
        } else if (!get_f32("attn_scale", 1.0f, c.attn_scale)) {
            return false;
        }
    }
    {
        auto it = meta.find("layer_kind");
        if (it == meta.end()) {
            c.layer_kind.assign(c.n_layers, c.n_experts > 0 ? 1 : 0);
        } else {
            if (it->second.type != 7 || it->second.bytes.size() != c.n_layers) {
                err = fmt("layer_kind must be a u8[] of %u entries", c.n_layers);
                return false;
            }
            c.layer_kind = it->second.bytes;
        }
    }
    for (uint8_t k : c.layer_kind) {
        if (k > 1) {
            err = "layer_kind entries must be 0 or 1";
            return false;
        }
        c.n_moe_layers += k;
    }
    if (c.n_moe_layers) {
        if (!c.n_experts || !c.top_k || c.top_k > c.n_experts || !c.expert_ffn_dim) {
            err = "MoE layers need n_experts >= 1, 1 <= top_k <= n_experts and expert_ffn_dim >= 1";
            return false;
        }
        if (!c.n_group || c.n_experts % c.n_group || !c.topk_group || c.topk_group > c.n_group ||
            c.top_k > c.topk_group * (c.n_experts / c.n_group)) {
            err = "n_group / topk_group do not fit n_experts and top_k";
            return false;
        }
    }

    // regions that must not overlap: preamble, metadata, directories, tensors, physical slabs
    std::vector<std::pair<uint64_t, uint64_t>> regions = {
        {0, kPreamble}, {meta_off, meta_bytes}, {tdir_off, n_tensors * kTensorEntry}, {edir_off, n_entries * kExpertEntry}};

    // ---- §4 tensor directory
    std::vector<uint8_t> td(n_tensors * kTensorEntry);
    if (!td.empty() && !read(tdir_off, td.data(), td.size(), err)) return false;
    c.tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors; i++) {
        const uint8_t *e = &td[i * kTensorEntry];
        CtTensor &t = c.tensors[i];
        if (e[kNameLen - 1] != 0 || e[0] == 0) {
            err = fmt("tensor entry %llu: name is empty or not NUL-terminated", (unsigned long long)i);
            return false;
        }
        t.name.assign(reinterpret_cast<const char *>(e), strnlen(reinterpret_cast<const char *>(e), kNameLen));
        t.dtype = rd32(e + 80);
        t.ndim = rd32(e + 84);
        for (int k = 0; k < 4; k++) t.shape[k] = rd32(e + 88 + 4 * k);
        t.off = rd64(e + 104);
        t.nbytes = rd64(e + 112);
        if (t.dtype > 6 || t.ndim < 1 || t.ndim > 4) {
            err = fmt("tensor %s: bad dtype %u or ndim %u", t.name.c_str(), t.dtype, t.ndim);
            return false;
        }
        uint64_t rows = 1;
        for (uint32_t k = 0; k < 4; k++) {
            if (t.shape[k] < 1 || (k >= t.ndim && t.shape[k] != 1)) {
                err = fmt("tensor %s: bad shape", t.name.c_str());
                return false;
            }
            if (k + 1 < t.ndim) rows *= t.shape[k];
        }
        const uint64_t rb = row_bytes_of(t.dtype, t.shape[t.ndim - 1]);
        if (!rb || t.nbytes != rows * rb) {
            err = fmt("tensor %s: %llu bytes do not match its shape and dtype", t.name.c_str(),
                      (unsigned long long)t.nbytes);
            return false;
        }
        if (t.off % kTensorAlign || !inside(t.off, t.nbytes)) {
            err = fmt("tensor %s: offset not 64-byte aligned or outside the file", t.name.c_str());
            return false;
        }
        if (!c.by_name.emplace(t.name, (size_t)i).second) {
            err = fmt("tensor %s appears twice", t.name.c_str());
            return false;
        }
        regions.push_back({t.off, t.nbytes});
    }

    // ---- §5 expert directory
    const uint64_t want_entries = c.n_experts ? (uint64_t)c.n_layers * c.n_experts : 0;
    if (n_entries != want_entries) {
        err = fmt("expert directory has %llu entries, expected n_layers * n_experts = %llu",
                  (unsigned long long)n_entries, (unsigned long long)want_entries);
        return false;
    }
    std::vector<uint8_t> ed(n_entries * kExpertEntry);
    if (!ed.empty() && !read(edir_off, ed.data(), ed.size(), err)) return false;
    c.experts.resize(n_entries);
    std::vector<size_t> moe_idx;
    for (uint64_t i = 0; i < n_entries; i++) {
        const uint8_t *e = &ed[i * kExpertEntry];
        CtExpert &x = c.experts[i];
        x.off = rd64(e);
        x.nbytes = rd64(e + 8);
        x.dtype = rd32(e + 16);
        x.flags = rd32(e + 20);
        const uint32_t layer = (uint32_t)(i / c.n_experts);
        if (!c.layer_kind[layer]) {
            if (x.nbytes) {
                err = fmt("expert entry %llu of dense layer %u has a slab", (unsigned long long)i, layer);
                return false;
            }
            continue;
        }
        if (x.dtype > 4) {
            err = fmt("expert entry %llu: slab dtype %u is not a float or block dtype", (unsigned long long)i, x.dtype);
            return false;
        }
        const uint64_t want = slab_size(x.dtype, c.d_model, c.expert_ffn_dim);
        if (!want || x.nbytes != want || x.off % kSlabAlign || !inside(x.off, x.nbytes)) {
            err = fmt("expert entry %llu (layer %u): slab of %llu bytes at %llu (expected %llu bytes, 4096-aligned, "
                      "inside the file)",
                      (unsigned long long)i, layer, (unsigned long long)x.nbytes, (unsigned long long)x.off,
                      (unsigned long long)want);
            return false;
        }
        moe_idx.push_back((size_t)i);
    }
    // entries sharing a slab: equal size and dtype, at most one without the aliased flag
    std::sort(moe_idx.begin(), moe_idx.end(),
              [&](size_t a, size_t b) { return c.experts[a].off < c.experts[b].off || (c.experts[a].off == c.experts[b].off && a < b); });
    for (size_t k = 0; k < moe_idx.size();) {
        size_t k1 = k + 1;
        const CtExpert &first = c.experts[moe_idx[k]];
        int owners = (first.flags & kFlagAliased) ? 0 : 1;
        while (k1 < moe_idx.size() && c.experts[moe_idx[k1]].off == first.off) {
            const CtExpert &x = c.experts[moe_idx[k1]];
            if (x.nbytes != first.nbytes || x.dtype != first.dtype) {
                err = fmt("expert entries %zu and %zu share a slab but differ in size or dtype", moe_idx[k], moe_idx[k1]);
                return false;
            }
            owners += (x.flags & kFlagAliased) ? 0 : 1;
            k1++;
        }
        if (owners > 1) {
            err = fmt("slab at %llu has %d entries without the aliased flag", (unsigned long long)first.off, owners);
            return false;
        }
        c.n_physical++;
        c.n_aliased += (int)(k1 - k - 1);
        regions.push_back({first.off, first.nbytes});
        c.expert_dtype = (k == 0 || c.expert_dtype == (int)first.dtype) ? (int)first.dtype : -2;
        k = k1;
    }
    if (c.expert_dtype < 0) c.expert_dtype = -1;

    std::sort(regions.begin(), regions.end());
    uint64_t end = 0;
    for (const auto &r : regions) {
        if (!r.second) continue;
        if (r.first < end) {
            err = fmt("regions overlap at byte %llu", (unsigned long long)r.first);
            return false;
        }
        end = r.first + r.second;
    }
    return true;
}

}  // namespace hx
