// loader.cu -- safetensors checkpoints straight into device memory.
//
// The reference reads a checkpoint by mmap'ing the file, parsing the JSON
// header and memcpy'ing every tensor into a host Tensor
// (src/loader/safetensors.cpp:71-131 open, 166-172 load_tensor_copy); its
// QwenModel then hands those host tensors to the backend.  Here the bytes go
// from the mapping to HBM through two pinned staging buffers: the host copy
// of one chunk into pinned memory overlaps the DMA of the previous chunk, so
// no pageable copy (which the driver would stage and serialise) is involved.
// Weights are then converted and tiled on the device by mrt_weight_upload /
// mrt_decoder_load, once.
//
// The header parser is this file's own: the subset of JSON a safetensors
// header uses (objects, arrays, strings with escapes, numbers, true / false /
// null), with the reference's rules -- "__metadata__" skipped, dtypes F16,
// BF16 and F32 accepted, anything else an error (safetensors.cpp:23-28,
// 33-69) -- plus bounds checks the reference leaves out: data offsets inside
// the file and a byte count equal to the shape's.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "ctx.h"

struct mrt_safetensors_s {
    struct Info {
        int dtype = MRT_FP16;
        std::vector<int64_t> shape;
        uint64_t offset = 0;  // from the start of the data section
        uint64_t bytes = 0;
    };
    std::string path;
    const uint8_t* map = nullptr;
    size_t file_bytes = 0;
    uint64_t data_start = 0;  // 8 + header length
    std::map<std::string, Info> tensors;  // sorted by name, like the reference's std::map
    std::vector<const std::string*> order;
};

namespace mrt {
namespace {

// ------------------------------------------------------------------ JSON subset

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    double num = 0.0;
    bool integral = false;
    uint64_t u = 0;  // the value when integral and non-negative
    bool neg = false;
    std::string str;
    std::vector<Json> items;                          // Array
    std::vector<std::pair<std::string, Json>> fields; // Object, in file order
};

class Parser {
public:
    Parser(const char* p, const char* end) : p_(p), end_(end) {}

    bool parse(Json* out, std::string* err) {
        if (!value(out, 0)) {
            *err = err_.empty() ? "malformed JSON" : err_;
            return false;
        }
        ws();
        if (p_ != end_) {
            *err = "trailing characters after the header object";
            return false;
        }
        return true;
    }

private:
    bool fail(const char* msg) {
        if (err_.empty()) err_ = msg;
        return false;
    }
    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* s) {
        const size_t n = std::strlen(s);
        if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, s, n) != 0) return fail("bad literal");
        p_ += n;
        return true;
    }
    static void utf8(uint32_t cp, std::string* s) {
        if (cp < 0x80) {
            s->push_back(static_cast<char>(cp));
        } else if (cp < 0x800) {
            s->push_back(static_cast<char>(0xC0 | (cp >> 6)));
            s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            s->push_back(static_cast<char>(0xE0 | (cp >> 12)));
            s->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else {
            s->push_back(static_cast<char>(0xF0 | (cp >> 18)));
            s->push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
            s->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            s->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        }
    }
    bool hex4(uint32_t* v) {
        if (end_ - p_ < 4) return fail("short \\u escape");
        *v = 0;
        for (int i = 0; i < 4; ++i) {
            const char c = *p_++;
            *v <<= 4;
            if (c >= '0' && c <= '9') *v |= static_cast<uint32_t>(c - '0');
            else if (c >= 'a' && c <= 'f') *v |= static_cast<uint32_t>(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') *v |= static_cast<uint32_t>(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string* s) {
        if (p_ >= end_ || *p_ != '"') return fail("expected a string");
        ++p_;
        while (p_ < end_ && *p_ != '"') {
            const char c = *p_++;
            if (static_cast<unsigned char>(c) < 0x20) return fail("control character in a string");
            if (c != '\\') {
                s->push_back(c);
                continue;
            }
            if (p_ >= end_) return fail("unterminated escape");
            const char e = *p_++;
            switch (e) {
                case '"': s->push_back('"'); break;
                case '\\': s->push_back('\\'); break;
                case '/': s->push_back('/'); break;
                case 'b': s->push_back('\b'); break;
                case 'f': s->push_back('\f'); break;
                case 'n': s->push_back('\n'); break;
                case 'r': s->push_back('\r'); break;
                case 't': s->push_back('\t'); break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(&cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
                        uint32_t lo;
                        if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') return fail("lone surrogate");
                        p_ += 2;
                        if (!hex4(&lo) || lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(cp, s);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p_ >= end_) return fail("unterminated string");
        ++p_;
        return true;
    }
    bool number(Json* out) {
        const char* s = p_;
        bool neg = false, frac = false;
        if (p_ < end_ && *p_ == '-') {
            neg = true;
            ++p_;
        }
        if (p_ >= end_ || *p_ < '0' || *p_ > '9') return fail("bad number");
        uint64_t u = 0;
        bool big = false;
        while (p_ < end_ && *p_ >= '0' && *p_ <= '9') {
            const uint64_t d = static_cast<uint64_t>(*p_ - '0');
            if (u > (UINT64_MAX - d) / 10) big = true;
            u = u * 10 + d;
            ++p_;
        }
        if (p_ < end_ && *p_ == '.') {
            frac = true;
            ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            frac = true;
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        out->kind = Json::Number;
        out->num = std::strtod(std::string(s, p_).c_str(), nullptr);
        out->integral = !frac && !big;
        out->neg = neg;
        out->u = u;
        return true;
    }
    bool value(Json* out, int depth) {
        if (depth > 64) return fail("JSON nested too deeply");
        ws();
        if (p_ >= end_) return fail("unexpected end of header");
        const char c = *p_;
        if (c == '{') {
            ++p_;
            out->kind = Json::Object;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            for (;;) {
                ws();
                std::string key;
                if (!string(&key)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
                ++p_;
                out->fields.emplace_back(std::move(key), Json());
                if (!value(&out->fields.back().second, depth + 1)) return false;
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            ++p_;
            out->kind = Json::Array;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            for (;;) {
                out->items.emplace_back();
                if (!value(&out->items.back(), depth + 1)) return false;
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            out->kind = Json::String;
            return string(&out->str);
        }
        if (c == 't') {
            out->kind = Json::Bool;
            out->num = 1;
            return lit("true");
        }
        if (c == 'f') {
            out->kind = Json::Bool;
            return lit("false");
        }
        if (c == 'n') {
            out->kind = Json::Null;
            return lit("null");
        }
        return number(out);
    }

    const char* p_;
    const char* end_;
    std::string err_;
};

const Json* field(const Json& obj, const char* key) {
    for (const auto& kv : obj.fields)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

bool as_u64(const Json& j, uint64_t* v) {
    if (j.kind != Json::Number || !j.integral || j.neg) return false;
    *v = j.u;
    return true;
}

size_t elem_size(int dt) { return dt == MRT_FP32 ? 4 : 2; }

// The reference's dtype table (safetensors.cpp:23-28).
int parse_dtype(const std::string& s, int* dt) {
    if (s == "F16") *dt = MRT_FP16;
    else if (s == "BF16") *dt = MRT_BF16;
    else if (s == "F32") *dt = MRT_FP32;
    else return set_error(MRT_ERR_DTYPE, "Unsupported dtype: " + s);
    return MRT_OK;
}

int parse_header(mrt_safetensors_s* f, const char* text, size_t len) {
    Json root;
    std::string err;
    Parser ps(text, text + len);
    if (!ps.parse(&root, &err)) return set_error(MRT_ERR_INVALID_ARG, "Failed to parse SafeTensors header JSON: " + err);
    if (root.kind != Json::Object) return set_error(MRT_ERR_INVALID_ARG, "SafeTensors header JSON must be an object");
    const uint64_t data_bytes = f->file_bytes - f->data_start;
    for (const auto& kv : root.fields) {
        const std::string& name = kv.first;
        if (name == "__metadata__") continue;
        const Json& t = kv.second;
        auto bad = [&](const std::string& why) {
            return set_error(MRT_ERR_INVALID_ARG, "Failed to parse tensor info for '" + name + "': " + why);
        };
        if (t.kind != Json::Object) return bad("tensor entry is not an object");
        const Json* dt = field(t, "dtype");
        const Json* sh = field(t, "shape");
        const Json* off = field(t, "data_offsets");
        if (dt == nullptr || dt->kind != Json::String) return bad("missing dtype");
        if (sh == nullptr || sh->kind != Json::Array) return bad("missing shape");
        if (off == nullptr || off->kind != Json::Array) return bad("missing data_offsets");
        mrt_safetensors_s::Info info;
        int rc = parse_dtype(dt->str, &info.dtype);
        if (rc != MRT_OK) return bad(mrt_last_error_string());
        uint64_t numel = 1;
        for (const Json& d : sh->items) {
            uint64_t v;
            if (!as_u64(d, &v) || v > (1ull << 40)) return bad("shape entries must be non-negative integers");
            info.shape.push_back(static_cast<int64_t>(v));
            numel = v == 0 ? 0 : (numel > (1ull << 62) / v ? (1ull << 62) : numel * v);
        }
        if (off->items.size() != 2) return bad("data_offsets must have exactly 2 elements");
        uint64_t a, b;
        if (!as_u64(off->items[0], &a) || !as_u64(off->items[1], &b) || b < a) return bad("bad data_offsets");
        if (b > data_bytes) return bad("data_offsets run past the end of the file");
        if (b - a != numel * elem_size(info.dtype)) return bad("data size does not match dtype and shape");
        info.offset = a;
        info.bytes = b - a;
        if (!f->tensors.emplace(name, std::move(info)).second) return bad("tensor listed twice");
    }
    for (const auto& kv : f->tensors) f->order.push_back(&kv.first);
    return MRT_OK;
}

const mrt_safetensors_s::Info* find(mrt_safetensors f, const char* name) {
    if (f == nullptr || name == nullptr) {
        set_error(MRT_ERR_INVALID_ARG, "NULL argument");
        return nullptr;
    }
    auto it = f->tensors.find(name);
    if (it == f->tensors.end()) {
        set_error(MRT_ERR_INVALID_ARG, std::string("no tensor '") + name + "' in " + f->path);
        return nullptr;
    }
    return &it->second;
}

// Two pinned chunks: the host copy into one overlaps the DMA out of the other.
constexpr size_t kStageChunk = 16u << 20;

struct Staging {
    void* pinned[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    ~Staging() {
        for (int i = 0; i < 2; ++i) {
            if (done[i]) {
                cudaEventSynchronize(done[i]);
                cudaEventDestroy(done[i]);
            }
            if (pinned[i]) cudaFreeHost(pinned[i]);
        }
    }
    int init() {
        for (int i = 0; i < 2; ++i) {
            cudaError_t e = cudaHostAlloc(&pinned[i], kStageChunk, cudaHostAllocDefault);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[i], cudaEventDisableTiming);
            if (e != cudaSuccess) return cuda_error(e, "allocating pinned staging");
        }
        return MRT_OK;
    }
    // bytes of host memory at src -> device memory at dst, ordered on s; returns
    // after every copy has been queued (the caller synchronises s).
    int to_device(void* dst, const uint8_t* src, uint64_t bytes, cudaStream_t s) {
        uint8_t* d = static_cast<uint8_t*>(dst);
        int slot = 0;
        for (uint64_t off = 0; off < bytes; off += kStageChunk, slot ^= 1) {
            const size_t n = static_cast<size_t>(std::min<uint64_t>(kStageChunk, bytes - off));
            cudaError_t e = cudaEventSynchronize(done[slot]);  // this chunk's last DMA has drained
            if (e != cudaSuccess) return cuda_error(e, "waiting for a staging buffer");
            std::memcpy(pinned[slot], src + off, n);
            e = cudaMemcpyAsync(d + off, pinned[slot], n, cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) e = cudaEventRecord(done[slot], s);
            if (e != cudaSuccess) return cuda_error(e, "copying a chunk to the device");
        }
        return MRT_OK;
    }
};

bool on_device(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Raw bytes of one tensor into a device buffer of at least info.bytes.
int stage_tensor(mrt_safetensors f, const mrt_safetensors_s::Info& info, void* dst_dev, Staging& st, cudaStream_t s) {
    return st.to_device(dst_dev, f->map + f->data_start + info.offset, info.bytes, s);
}

// Names the decoder takes (the reference's QwenModel::load_weights,
// qwen_model.cpp:336-353, and the blocks' loaders it calls); every other
// tensor of a checkpoint is ignored there too.
bool decoder_takes(const std::string& name, int64_t n_layers) {
    if (name == "model.embed_tokens.weight" || name == "lm_head.weight" || name == "model.norm.weight") return true;
    static const char* kPrefix = "model.layers.";
    if (name.compare(0, std::strlen(kPrefix), kPrefix) != 0) return false;
    size_t i = std::strlen(kPrefix);
    int64_t li = 0;
    size_t digits = 0;
    while (i < name.size() && name[i] >= '0' && name[i] <= '9' && digits < 9) {
        li = li * 10 + (name[i] - '0');
        ++i;
        ++digits;
    }
    if (digits == 0 || i >= name.size() || name[i] != '.' || li >= n_layers) return false;
    static const char* kSuffixes[] = {"input_layernorm.weight", "post_attention_layernorm.weight",
                                      "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                                      "self_attn.v_proj.weight", "self_attn.q_proj.bias",
                                      "self_attn.k_proj.bias",   "self_attn.v_proj.bias",
                                      "self_attn.o_proj.weight", "mlp.gate_proj.weight",
                                      "mlp.up_proj.weight",      "mlp.down_proj.weight"};
    const std::string suf = name.substr(i + 1);
    for (const char* s : kSuffixes)
        if (suf == s) return true;
    return false;
}

}  // namespace
}  // namespace mrt

using namespace mrt;

extern "C" int mrt_safetensors_open(const char* path, mrt_safetensors* out) {
    clear_error();
    if (path == nullptr || out == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return set_error(MRT_ERR_INVALID_ARG, std::string("Failed to open file: ") + path);
    struct stat st{};
    if (fstat(fd, &st) < 0) {
        ::close(fd);
        return set_error(MRT_ERR_INVALID_ARG, std::string("Failed to stat file: ") + path);
    }
    auto* f = new mrt_safetensors_s();
    f->path = path;
    f->file_bytes = static_cast<size_t>(st.st_size);
    if (f->file_bytes < 8) {
        ::close(fd);
        delete f;
        return set_error(MRT_ERR_INVALID_ARG, std::string("File too small to be SafeTensors: ") + path);
    }
    void* m = mmap(nullptr, f->file_bytes, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        delete f;
        return set_error(MRT_ERR_INVALID_ARG, std::string("Failed to mmap file: ") + path);
    }
    f->map = static_cast<const uint8_t*>(m);
    uint64_t hlen = 0;
    std::memcpy(&hlen, f->map, 8);
    if (hlen > f->file_bytes - 8) {
        munmap(m, f->file_bytes);
        delete f;
        return set_error(MRT_ERR_INVALID_ARG, std::string("Invalid header size in SafeTensors file: ") + path);
    }
    f->data_start = 8 + hlen;
    const int rc = parse_header(f, reinterpret_cast<const char*>(f->map + 8), static_cast<size_t>(hlen));
    if (rc != MRT_OK) {
        munmap(m, f->file_bytes);
        delete f;
        return rc;
    }
    *out = f;
    return MRT_OK;
}

extern "C" int mrt_safetensors_close(mrt_safetensors f) {
    if (f == nullptr) return MRT_OK;
    if (f->map) munmap(const_cast<uint8_t*>(f->map), f->file_bytes);
    delete f;
    return MRT_OK;
}

extern "C" int mrt_safetensors_count(mrt_safetensors f, int64_t* n) {
    clear_error();
    if (f == nullptr || n == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    *n = static_cast<int64_t>(f->order.size());
    return MRT_OK;
}

extern "C" int mrt_safetensors_name(mrt_safetensors f, int64_t i, const char** name) {
    clear_error();
    if (f == nullptr || name == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (i < 0 || i >= static_cast<int64_t>(f->order.size())) return set_error(MRT_ERR_INVALID_ARG, "tensor index out of range");
    *name = f->order[static_cast<size_t>(i)]->c_str();
    return MRT_OK;
}

extern "C" int mrt_safetensors_info(mrt_safetensors f, const char* name, int* dtype, int* ndim, int64_t* shape,
                                    uint64_t* nbytes) {
    clear_error();
    const auto* info = find(f, name);
    if (info == nullptr) return MRT_ERR_INVALID_ARG;
    if (dtype) *dtype = info->dtype;
    if (ndim) *ndim = static_cast<int>(info->shape.size());
    if (shape)
        for (size_t i = 0; i < info->shape.size() && i < 8; ++i) shape[i] = info->shape[i];
    if (nbytes) *nbytes = info->bytes;
    return MRT_OK;
}

extern "C" int mrt_safetensors_read(mrt_safetensors f, const char* name, void* dst, uint64_t dst_bytes, void* stream) {
    clear_error();
    const auto* info = find(f, name);
    if (info == nullptr) return MRT_ERR_INVALID_ARG;
    if (dst == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL destination");
    if (dst_bytes < info->bytes)
        return set_error(MRT_ERR_SHAPE, std::string(name) + ": needs " + std::to_string(info->bytes) + " bytes, got " +
                                            std::to_string(dst_bytes));
    if (!on_device(dst)) {
        std::memcpy(dst, f->map + f->data_start + info->offset, info->bytes);
        return MRT_OK;
    }
    if (!current_ctx()) return MRT_ERR_CUDA;
    Staging st;
    int rc = st.init();
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (rc == MRT_OK) rc = stage_tensor(f, *info, dst, st, s);
    if (rc != MRT_OK) return rc;
    const cudaError_t e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? MRT_OK : cuda_error(e, "waiting for the staged copy");
}

extern "C" int mrt_safetensors_upload_weight(mrt_safetensors f, const char* name, const int64_t* row_ranges,
                                             int64_t n_ranges, int64_t k0, int64_t k1, void* stream, mrt_weight* out) {
    clear_error();
    const auto* info = find(f, name);
    if (info == nullptr) return MRT_ERR_INVALID_ARG;
    if (out == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL output");
    if (info->shape.size() != 2) return set_error(MRT_ERR_SHAPE, std::string(name) + ": a weight is 2-D [N, K]");
    if (!current_ctx()) return MRT_ERR_CUDA;
    void* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, std::max<uint64_t>(info->bytes, 16));
    if (e != cudaSuccess) return cuda_error(e, "allocating the upload buffer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int rc;
    {
        Staging st;
        rc = st.init();
        if (rc == MRT_OK) rc = stage_tensor(f, *info, tmp, st, s);
    }
    if (rc == MRT_OK)
        rc = mrt_weight_upload(tmp, info->dtype, 1, info->shape[0], info->shape[1], row_ranges, n_ranges, k0, k1, stream,
                               out);
    e = cudaStreamSynchronize(s);  // the upload has read tmp
    cudaFree(tmp);
    if (rc == MRT_OK && e != cudaSuccess) rc = cuda_error(e, "waiting for the weight upload");
    return rc;
}

extern "C" int mrt_decoder_load_safetensors(mrt_decoder d, mrt_safetensors f, int64_t* n_loaded) {
    clear_error();
    if (d == nullptr || f == nullptr) return set_error(MRT_ERR_INVALID_ARG, "NULL argument");
    if (n_loaded) *n_loaded = 0;
    const int64_t layers = decoder_layer_count(d);
    int rc = MRT_OK;
    if (!current_ctx()) return MRT_ERR_CUDA;
    uint64_t biggest = 16;
    for (const auto& kv : f->tensors)
        if (decoder_takes(kv.first, layers)) biggest = std::max(biggest, kv.second.bytes);
    void* tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, biggest);
    if (e != cudaSuccess) return cuda_error(e, "allocating the checkpoint staging buffer");
    cudaStream_t s = nullptr;
    e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        cudaFree(tmp);
        return cuda_error(e, "creating the loader stream");
    }
    {
        Staging st;
        rc = st.init();
        int64_t n = 0;
        for (const std::string* name : f->order) {
            if (rc != MRT_OK) break;
            if (!decoder_takes(*name, layers)) continue;
            const auto& info = f->tensors.at(*name);
            if (info.shape.empty() || info.shape.size() > 2) {
                rc = set_error(MRT_ERR_SHAPE, *name + ": expected a 1-D or 2-D tensor");
                break;
            }
            if ((rc = stage_tensor(f, info, tmp, st, s)) != MRT_OK) break;
            e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) {
                rc = cuda_error(e, "waiting for a staged tensor");
                break;
            }
            const int64_t rows = info.shape[0], cols = info.shape.size() == 2 ? info.shape[1] : 1;
            // mrt_decoder_load orders itself after this device source and
            // has read it when the device next synchronises.
            if ((rc = mrt_decoder_load(d, name->c_str(), tmp, info.dtype, 1, rows, cols)) != MRT_OK) break;
            e = cudaDeviceSynchronize();
            if (e != cudaSuccess) {
                rc = cuda_error(e, "waiting for the decoder's copy of a tensor");
                break;
            }
            ++n;
        }
        if (n_loaded) *n_loaded = n;
    }
    cudaStreamDestroy(s);
    cudaFree(tmp);
    return rc;
}
