// GGUF expert-slice reader: the host side of loading a layer's experts from a
// (possibly sharded) GGUF checkpoint.
//
// Follows the reference's load_gguf_experts (tools/engine/gguf_experts.cpp:45-140,
// LoadedExperts in gguf_experts.hpp:14-20): shards "<stem>-00001-of-NNNNN.gguf"
// (cpp:27-41), tensors blk.L.ffn_{gate,up,down}_exps.{weight,bias}, each tensor in one
// shard only, the selected experts' byte slices (stride = tensor bytes / experts) plus
// their fp32 values, and the same validation.  The reference parses the container
// with ggml's gguf reader (a dependency absent here); this file reads the GGUF v2/v3
// container directly: header, key/value pairs (only general.alignment is used),
// tensor infos, aligned data section.  Every read is bounds-checked against the file.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "umsx_internal.h"

namespace umsx {
namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF"
constexpr int kTypeF32 = 0, kTypeF16 = 1, kTypeQ8_0 = 8, kTypeBF16 = 30, kTypeMXFP4 = 39;

struct TensorInfo {
    int64_t ne[4] = {1, 1, 1, 1};
    int type = -1;
    uint64_t offset = 0;  // from the data section start
};

// Block size (elements) and bytes per block of the types this reader decodes.
bool type_geometry(int type, int64_t &blck, int64_t &bytes) {
    switch (type) {
        case kTypeF32: blck = 1; bytes = 4; return true;
        case kTypeF16: blck = 1; bytes = 2; return true;
        case kTypeBF16: blck = 1; bytes = 2; return true;
        case kTypeQ8_0: blck = 32; bytes = 34; return true;
        case kTypeMXFP4: blck = 32; bytes = 17; return true;
        default: return false;
    }
}

const char *type_name(int type) {
    switch (type) {
        case kTypeF32: return "f32";
        case kTypeF16: return "f16";
        case kTypeBF16: return "bf16";
        case kTypeQ8_0: return "q8_0";
        case kTypeMXFP4: return "mxfp4";
        default: return "unsupported";
    }
}

class Reader {
  public:
    explicit Reader(const std::string &path) : in_(path, std::ios::binary) {
        if (in_) {
            in_.seekg(0, std::ios::end);
            size_ = (uint64_t)in_.tellg();
            in_.seekg(0);
        }
    }
    bool ok() const { return (bool)in_; }
    uint64_t size() const { return size_; }
    uint64_t pos() { return (uint64_t)in_.tellg(); }
    bool bytes(void *dst, uint64_t n) {
        if (!in_ || n > size_ || pos() > size_ - n) return false;
        in_.read(static_cast<char *>(dst), (std::streamsize)n);
        return (bool)in_;
    }
    template <class T>
    bool get(T &v) { return bytes(&v, sizeof(T)); }
    bool skip(uint64_t n) {
        if (!in_ || n > size_ || pos() > size_ - n) return false;
        in_.seekg((std::streamoff)n, std::ios::cur);
        return (bool)in_;
    }
    bool str(std::string &s, uint64_t max_len = 1u << 20) {
        uint64_t n;
        if (!get(n) || n > max_len) return false;
        s.resize(n);
        return n == 0 || bytes(&s[0], n);
    }
    bool seek(uint64_t off) {
        if (!in_ || off > size_) return false;
        in_.seekg((std::streamoff)off);
        return (bool)in_;
    }

  private:
    std::ifstream in_;
    uint64_t size_ = 0;
};

// Skips one key/value payload of GGUF value type `vt`; reads general.alignment into *align.
bool skip_value(Reader &r, uint32_t vt, int depth, uint64_t *as_uint) {
    static const int kScalar[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (vt > 12) return false;
    if (vt == 8) {  // string
        std::string s;
        return r.str(s);
    }
    if (vt == 9) {  // array
        if (depth > 2) return false;
        uint32_t et;
        uint64_t n;
        if (!r.get(et) || !r.get(n) || et > 12) return false;
        if (et != 8 && et != 9) return n <= r.size() && r.skip(n * (uint64_t)kScalar[et]);
        if (n > r.size()) return false;
        for (uint64_t i = 0; i < n; ++i)
            if (!skip_value(r, et, depth + 1, nullptr)) return false;
        return true;
    }
    uint64_t v = 0;
    if (!r.bytes(&v, (uint64_t)kScalar[vt])) return false;
    if (as_uint) *as_uint = v;
    return true;
}

struct GgufFile {
    uint64_t file_size = 0, data_offset = 0;
    std::map<std::string, TensorInfo> tensors;
};

std::string parse_gguf(const std::string &path, GgufFile &f) {
    Reader r(path);
    if (!r.ok()) return "GGUF shard missing or not readable: " + path;
    f.file_size = r.size();
    uint32_t magic, version;
    uint64_t n_tensors, n_kv;
    if (!r.get(magic) || magic != kGgufMagic) return "not a GGUF file: " + path;
    if (!r.get(version) || (version != 2 && version != 3)) return "unsupported GGUF version in " + path;
    if (!r.get(n_tensors) || !r.get(n_kv) || n_tensors > (1u << 24) || n_kv > (1u << 24))
        return "GGUF header could not be read: " + path;
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key;
        uint32_t vt;
        if (!r.str(key) || !r.get(vt)) return "GGUF metadata could not be read: " + path;
        uint64_t v = 0;
        if (!skip_value(r, vt, 0, &v)) return "GGUF metadata could not be read: " + path;
        if (key == "general.alignment") {
            if (vt != 4 || v == 0 || (v & (v - 1)) || v > 4096) return "invalid general.alignment in " + path;
            alignment = v;
        }
    }
    for (uint64_t i = 0; i < n_tensors; ++i) {
        std::string name;
        uint32_t n_dims;
        TensorInfo t;
        if (!r.str(name) || !r.get(n_dims) || n_dims < 1 || n_dims > 4) return "GGUF tensor info could not be read: " + path;
        for (uint32_t d = 0; d < n_dims; ++d) {
            uint64_t ne;
            if (!r.get(ne) || ne == 0 || ne > (1ull << 40)) return "invalid GGUF tensor shape: " + name;
            t.ne[d] = (int64_t)ne;
        }
        // every size below is a product of these extents: bound the element count so that no
        // product (nor its byte count) can overflow
        int64_t count = 1;
        for (int d = 0; d < 4; ++d) {
            if (t.ne[d] > ((int64_t)1 << 56) / count) return "invalid GGUF tensor shape (element count overflows): " + name;
            count *= t.ne[d];
        }
        uint32_t type;
        if (!r.get(type) || !r.get(t.offset)) return "GGUF tensor info could not be read: " + path;
        t.type = (int)type;
        if (f.tensors.count(name)) return "duplicate GGUF tensor " + name + " in " + path;
        f.tensors.emplace(name, t);
    }
    const uint64_t end = r.pos();
    f.data_offset = (end + alignment - 1) / alignment * alignment;
    if (f.data_offset > f.file_size) return "GGUF data section exceeds shard: " + path;
    return "";
}

std::vector<std::string> shard_paths(const std::string &first) {
    std::vector<std::string> out{first};
    const size_t slash = first.find_last_of('/');
    const std::string dir = slash == std::string::npos ? "" : first.substr(0, slash + 1);
    const std::string name = slash == std::string::npos ? first : first.substr(slash + 1);
    // <stem>-00001-of-NNNNN.gguf
    const std::string tail = ".gguf";
    if (name.size() < 20 || name.compare(name.size() - tail.size(), tail.size(), tail) != 0) return out;
    const std::string core = name.substr(0, name.size() - tail.size());  // <stem>-00001-of-NNNNN
    if (core.size() < 15) return out;
    const std::string suf = core.substr(core.size() - 15);  // -00001-of-NNNNN
    auto digits = [](const std::string &s) {
        for (char c : s)
            if (c < '0' || c > '9') return false;
        return true;
    };
    if (suf.compare(0, 7, "-00001-") != 0 || suf.compare(7, 3, "of-") != 0 || !digits(suf.substr(10, 5))) return out;
    const int count = std::stoi(suf.substr(10, 5));
    if (count < 1 || count > 100) return {};  // the caller reports the invalid count
    const std::string stem = core.substr(0, core.size() - 15);
    for (int i = 2; i <= count; ++i) {
        char buf[32];
        std::snprintf(buf, sizeof(buf), "-%05d-of-%05d.gguf", i, count);
        out.push_back(dir + stem + buf);
    }
    return out;
}

float half_to_float(uint16_t h) {
    const uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31, m = h & 1023;
    uint32_t bits;
    if (e == 0) {
        if (m == 0) {
            bits = s;
        } else {  // subnormal: m * 2^-24, exact in fp32
            float v = (float)m * 0x1p-24f;
            std::memcpy(&bits, &v, 4);
            bits |= s;
        }
    } else if (e == 31) {
        bits = s | 0x7f800000u | (m << 13);
    } else {
        bits = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

float bf16_to_float(uint16_t b) {
    const uint32_t bits = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// e8m0 scale of an MXFP4 block, halved (the e2m1 values below are doubled): 2^(e - 128).
float e8m0_half(uint8_t e) {
    uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// fp32 values of n elements of a row of `type` (n a multiple of the block size).
void dequantize(int type, const uint8_t *src, int64_t n, float *dst) {
    static const int8_t kE2m1x2[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
    switch (type) {
        case kTypeF32: std::memcpy(dst, src, (size_t)n * 4); break;
        case kTypeF16:
            for (int64_t i = 0; i < n; ++i) dst[i] = half_to_float((uint16_t)(src[2 * i] | src[2 * i + 1] << 8));
            break;
        case kTypeBF16:
            for (int64_t i = 0; i < n; ++i) dst[i] = bf16_to_float((uint16_t)(src[2 * i] | src[2 * i + 1] << 8));
            break;
        case kTypeQ8_0:
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t *blk = src + b * 34;
                const float d = half_to_float((uint16_t)(blk[0] | blk[1] << 8));
                for (int j = 0; j < 32; ++j) dst[b * 32 + j] = d * (float)(int8_t)blk[2 + j];
            }
            break;
        case kTypeMXFP4:  // element j < 16: low nibble of byte j; element 16 + j: its high nibble
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t *blk = src + b * 17;
                const float d = e8m0_half(blk[0]);
                for (int j = 0; j < 16; ++j) {
                    dst[b * 32 + j] = (float)kE2m1x2[blk[1 + j] & 15] * d;
                    dst[b * 32 + 16 + j] = (float)kE2m1x2[blk[1 + j] >> 4] * d;
                }
            }
            break;
        default: break;
    }
}

struct Found {
    std::string shard;
    GgufFile *file = nullptr;
    TensorInfo t;
};

}  // namespace

std::string gguf_load_experts(const std::string &first_shard, int layer, const std::vector<uint32_t> &ids,
                              bool dequant, bool bounded, GgufExperts &out) {
    if (layer < 0 || layer >= 4096 || ids.empty() || (bounded && ids.size() > 16) ||
        std::set<uint32_t>(ids.begin(), ids.end()).size() != ids.size())
        return "invalid layer or selected expert IDs";
    const std::vector<std::string> shards = shard_paths(first_shard);
    if (shards.empty()) return "invalid GGUF shard count";
    std::vector<GgufFile> files(shards.size());
    const std::string prefix = "blk." + std::to_string(layer) + ".ffn_";
    static const char *kParts[3] = {"gate", "up", "down"};
    Found found[3][2];  // [part][weight, bias]
    bool have[3][2] = {};
    for (size_t s = 0; s < shards.size(); ++s) {
        if (std::string err = parse_gguf(shards[s], files[s]); !err.empty()) return err;
        for (int p = 0; p < 3; ++p)
            for (int k = 0; k < 2; ++k) {
                const std::string name = prefix + kParts[p] + "_exps." + (k ? "bias" : "weight");
                auto it = files[s].tensors.find(name);
                if (it == files[s].tensors.end()) continue;
                if (have[p][k]) return "duplicate GGUF expert tensor across shards: " + name;
                have[p][k] = true;
                found[p][k] = Found{shards[s], &files[s], it->second};
            }
    }
    const uint32_t max_id = *std::max_element(ids.begin(), ids.end());
    for (int p = 0; p < 3; ++p) {
        if (!have[p][0]) return "required separate expert tensors are missing";
        for (int k = 0; k < 2; ++k) {
            if (!have[p][k]) continue;
            const TensorInfo &t = found[p][k].t;
            const std::string name = prefix + kParts[p] + "_exps." + (k ? "bias" : "weight");
            if (t.ne[3] != 1) return "invalid GGUF expert tensor shape: " + name;
            const int64_t count = k == 0 ? t.ne[2] : t.ne[1];
            if (count <= 0 || count > 65536 || (k == 1 && t.ne[2] != 1) || (int64_t)max_id >= count)
                return "GGUF expert ID outside tensor: " + name;
            int64_t blck, bb;
            if (!type_geometry(t.type, blck, bb))
                return std::string("GGUF expert quantization has no dequantizer: ") + name + " type " + std::to_string(t.type);
            if (t.ne[0] % blck) return "GGUF row length not a multiple of the block size: " + name;
            const int64_t elements = t.ne[0] * t.ne[1] * t.ne[2] / count;
            if (bounded && (uint64_t)elements > (32ull * 1024 * 1024) / ids.size())
                return "selected expert tensor exceeds bounded size: " + name;
            const uint64_t bytes = (uint64_t)(t.ne[0] * t.ne[1] * t.ne[2] / blck) * (uint64_t)bb;
            if (bytes % (uint64_t)count) return "nonuniform GGUF expert tensor layout: " + name;
            const uint64_t stride = bytes / (uint64_t)count;
            const GgufFile &f = *found[p][k].file;
            if (t.offset > f.file_size - f.data_offset) return "GGUF tensor offset exceeds shard: " + name;
            const uint64_t off = f.data_offset + t.offset;
            if (bytes > f.file_size - off) return "GGUF tensor exceeds shard: " + name;
            if (k == 1 && t.type != kTypeF32 && t.type != kTypeF16 && t.type != kTypeBF16)
                return "GGUF expert bias must be f32, f16 or bf16: " + name;
            std::ifstream in(found[p][k].shard, std::ios::binary);
            if (!in) return "GGUF shard could not be opened: " + found[p][k].shard;
            std::vector<uint8_t> slice(stride);
            std::vector<uint8_t> &packed = out.packed[p];
            std::vector<float> &vals = k ? out.bias[p] : out.values[p];
            if (k == 0) {
                out.type[p] = t.type;
                out.stride[p] = stride;
                out.shape[p][0] = t.ne[0];
                out.shape[p][1] = t.ne[1];
                out.shape[p][2] = t.ne[2];
                packed.assign(stride * ids.size(), 0);
            } else {
                out.has_bias[p] = true;
                out.bias_len[p] = t.ne[0];
            }
            if (k == 1 || dequant) vals.assign((size_t)elements * ids.size(), 0.0f);
            for (size_t i = 0; i < ids.size(); ++i) {
                in.seekg((std::streamoff)(off + stride * ids[i]));
                in.read(reinterpret_cast<char *>(slice.data()), (std::streamsize)stride);
                if (!in) return "GGUF expert slice could not be read: " + name;
                if (k == 0) std::memcpy(packed.data() + i * stride, slice.data(), stride);
                if (k == 1 || dequant) dequantize(t.type, slice.data(), elements, vals.data() + i * (size_t)elements);
            }
        }
    }
    const int64_t *g = out.shape[0], *u = out.shape[1], *dn = out.shape[2];
    if (g[0] != u[0] || g[1] != u[1] || g[2] != u[2] || dn[0] != g[1] || dn[1] != g[0] || dn[2] != g[2])
        return "incompatible expert projection shapes";
    out.hidden = (int)g[0];
    out.intermediate = (int)g[1];
    out.count = (int)g[2];
    out.n_ids = (int)ids.size();
    for (int p = 0; p < 3; ++p)
        if (out.has_bias[p] && out.bias_len[p] != (p == 2 ? g[0] : g[1])) return "incompatible expert bias shape";
    return "";
}

std::string gguf_load_router(const std::string &first_shard, int layer, std::vector<float> &w, int64_t shape[2],
                             std::vector<float> &b, bool &has_b) {
    const std::vector<std::string> shards = shard_paths(first_shard);
    if (shards.empty()) return "invalid GGUF shard count";
    const std::string names[2] = {"blk." + std::to_string(layer) + ".ffn_gate_inp.weight",
                                  "blk." + std::to_string(layer) + ".ffn_gate_inp.bias"};
    bool have[2] = {};
    has_b = false;
    for (const std::string &path : shards) {
        GgufFile f;
        if (std::string err = parse_gguf(path, f); !err.empty()) return err;
        for (int k = 0; k < 2; ++k) {
            auto it = f.tensors.find(names[k]);
            if (it == f.tensors.end()) continue;
            if (have[k]) return "duplicate GGUF router tensor across shards: " + names[k];
            have[k] = true;
            const TensorInfo &t = it->second;
            if (t.type != kTypeF32 && t.type != kTypeF16 && t.type != kTypeBF16)
                return std::string("GGUF router tensor must be f32, f16 or bf16: ") + names[k] + " is " + type_name(t.type);
            if (t.ne[2] != 1 || t.ne[3] != 1 || (k == 1 && t.ne[1] != 1)) return "invalid GGUF router shape: " + names[k];
            int64_t blck, bb;
            type_geometry(t.type, blck, bb);
            const int64_t n = t.ne[0] * t.ne[1];
            const uint64_t bytes = (uint64_t)n * (uint64_t)bb;
            if (t.offset > f.file_size - f.data_offset || bytes > f.file_size - f.data_offset - t.offset)
                return "GGUF tensor exceeds shard: " + names[k];
            std::vector<uint8_t> raw(bytes);
            std::ifstream in(path, std::ios::binary);
            in.seekg((std::streamoff)(f.data_offset + t.offset));
            in.read(reinterpret_cast<char *>(raw.data()), (std::streamsize)bytes);
            if (!in) return "GGUF router tensor could not be read: " + names[k];
            std::vector<float> &dst = k ? b : w;
            dst.assign((size_t)n, 0.0f);
            dequantize(t.type, raw.data(), n, dst.data());
            if (k == 0) {
                shape[0] = t.ne[0];
                shape[1] = t.ne[1];
            } else {
                has_b = true;
            }
        }
    }
    if (!have[0]) return "GGUF router tensor missing: " + names[0];
    if (has_b && (int64_t)b.size() != shape[1]) return "incompatible GGUF router bias shape";
    return "";
}

}  // namespace umsx
