// yk_loader.cu -- checkpoints at the boundary.
//
//  * yk_safetensors_*: the .safetensors reader (S/SafetensorsReader.swift:18-128):
//    mmap the file, parse the 8-byte little-endian header length and the JSON
//    header, expose each tensor's dtype, shape and mapped bytes.  Unlike the
//    reference it validates the header (offsets inside the data block, byte
//    count = product(shape) x element size, no duplicate names) and rejects a
//    malformed file with YK_ERR_ARG instead of trusting it.
//  * yk_model_load_tensor: ModelLoader.loadLinearLayer (S/ModelLoader.swift:9-72)
//    for this module's device layout: the source may be F32, F16 (the reference's
//    two branches) or BF16, in the checkpoint's [out x in] or the reference's
//    [in x out] layout; conversion and transposition run on the device.  A
//    tensor-parallel shard takes its window of the full tensor.
//  * yk_model_load_safetensors: every tensor of a (sharded) checkpoint under the
//    Hugging Face Llama / Gemma names.
//
// Host pipeline: each tensor streams through two pinned staging slots; while the
// device converts slot i (H2D copy + one kernel), the host gathers the next
// chunk's rows into slot i^1.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <cuda_fp16.h>

#include "yk_common.cuh"
#include "yk_internal.h"

// ---------------------------------------------------------------------------
// JSON (the header only): objects, arrays, strings, numbers, literals.
// ---------------------------------------------------------------------------
namespace {

struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    bool is_int = false;  // an integer literal that fits int64
    long long i = 0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
};

class JParser {
  public:
    JParser(const char* p, size_t n) : p_(p), end_(p + n) {}
    bool parse(JVal& out) {
        if (!value(out, 0)) return false;
        ws();
        return p_ == end_;
    }

  private:
    static constexpr int kMaxDepth = 32;
    const char* p_;
    const char* end_;

    void ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if ((size_t)(end_ - p_) < n || std::memcmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void utf8(std::string& s, unsigned cp) {
        if (cp < 0x80) {
            s += (char)cp;
        } else if (cp < 0x800) {
            s += (char)(0xC0 | (cp >> 6));
            s += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            s += (char)(0xE0 | (cp >> 12));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        } else {
            s += (char)(0xF0 | (cp >> 18));
            s += (char)(0x80 | ((cp >> 12) & 0x3F));
            s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        }
    }
    // One raw multi-byte character whose lead byte c was just consumed, appended to
    // s if it is well-formed UTF-8 (RFC 3629: no overlong forms, no surrogates,
    // nothing above U+10FFFF) -- JSON text is UTF-8, and names end up as C strings
    // that callers decode as UTF-8.
    bool utf8_seq(unsigned char c, std::string& s) {
        int n;
        unsigned char lo = 0x80, hi = 0xBF;  // range of the second byte
        if (c >= 0xC2 && c <= 0xDF) n = 1;
        else if (c >= 0xE0 && c <= 0xEF) {
            n = 2;
            if (c == 0xE0) lo = 0xA0;
            if (c == 0xED) hi = 0x9F;
        } else if (c >= 0xF0 && c <= 0xF4) {
            n = 3;
            if (c == 0xF0) lo = 0x90;
            if (c == 0xF4) hi = 0x8F;
        } else {
            return false;
        }
        if (end_ - p_ < n) return false;
        for (int k = 0; k < n; ++k) {
            const unsigned char b = (unsigned char)p_[k];
            if (k == 0 ? (b < lo || b > hi) : (b < 0x80 || b > 0xBF)) return false;
        }
        s += (char)c;
        s.append(p_, (size_t)n);
        p_ += n;
        return true;
    }
    bool hex4(unsigned& v) {
        if (end_ - p_ < 4) return false;
        v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (unsigned)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (unsigned)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (unsigned)(c - 'A' + 10);
            else return false;
        }
        return true;
    }
    bool str(std::string& s) {
        if (p_ >= end_ || *p_ != '"') return false;
        ++p_;
        while (p_ < end_) {
            const unsigned char c = (unsigned char)*p_++;
            if (c == '"') return true;
            if (c < 0x20) return false;
            if (c >= 0x80) {
                if (!utf8_seq(c, s)) return false;
                continue;
            }
            if (c != '\\') {
                s += (char)c;
                continue;
            }
            if (p_ >= end_) return false;
            const char e = *p_++;
            switch (e) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    unsigned cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // surrogate pair
                        unsigned lo;
                        if (end_ - p_ < 6 || p_[0] != '\\' || p_[1] != 'u') return false;
                        p_ += 2;
                        if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return false;
                    }
                    utf8(s, cp);
                    break;
                }
                default: return false;
            }
        }
        return false;
    }
    bool num(JVal& v) {
        const char* b = p_;
        if (p_ < end_ && *p_ == '-') ++p_;
        if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
        if (*p_ == '0') ++p_;
        else
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        bool integral = true;
        if (p_ < end_ && *p_ == '.') {
            integral = false;
            ++p_;
            if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            integral = false;
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= end_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        v.kind = JVal::NUM;
        if (integral) {
            // exact int64 (shapes and byte offsets); larger magnitudes are not integers here
            const bool neg = *b == '-';
            unsigned long long acc = 0;
            bool ok = true;
            for (const char* q = b + (neg ? 1 : 0); q < p_; ++q) {
                const unsigned d = (unsigned)(*q - '0');
                if (acc > (0x7FFFFFFFFFFFFFFFull - d) / 10) {
                    ok = false;
                    break;
                }
                acc = acc * 10 + d;
            }
            v.is_int = ok;
            v.i = ok ? (neg ? -(long long)acc : (long long)acc) : 0;
        }
        return true;
    }
    bool value(JVal& v, int depth) {
        if (depth > kMaxDepth) return false;
        ws();
        if (p_ >= end_) return false;
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v.kind = JVal::OBJ;
            ws();
            if (p_ < end_ && *p_ == '}') {
                ++p_;
                return true;
            }
            for (;;) {
                ws();
                std::pair<std::string, JVal> kv;
                if (!str(kv.first)) return false;
                ws();
                if (p_ >= end_ || *p_ != ':') return false;
                ++p_;
                if (!value(kv.second, depth + 1)) return false;
                v.obj.push_back(std::move(kv));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == '}') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '[') {
            ++p_;
            v.kind = JVal::ARR;
            ws();
            if (p_ < end_ && *p_ == ']') {
                ++p_;
                return true;
            }
            for (;;) {
                JVal e;
                if (!value(e, depth + 1)) return false;
                v.arr.push_back(std::move(e));
                ws();
                if (p_ < end_ && *p_ == ',') {
                    ++p_;
                    continue;
                }
                if (p_ < end_ && *p_ == ']') {
                    ++p_;
                    return true;
                }
                return false;
            }
        }
        if (c == '"') {
            v.kind = JVal::STR;
            return str(v.s);
        }
        if (c == 't' && lit("true")) {
            v.kind = JVal::BOOL;
            v.b = true;
            return true;
        }
        if (c == 'f' && lit("false")) {
            v.kind = JVal::BOOL;
            return true;
        }
        if (c == 'n' && lit("null")) {
            v.kind = JVal::NUL;
            return true;
        }
        return num(v);
    }
};

const JVal* member(const JVal& o, const char* key) {
    for (const auto& kv : o.obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

// The safetensors dtype names; code = YK_DTYPE_* where this module converts it, else -1.
struct DtypeName {
    const char* name;
    int code;
    int bytes;
};
constexpr DtypeName kDtypes[] = {
    {"F32", YK_DTYPE_F32, 4}, {"BF16", YK_DTYPE_BF16, 2}, {"F16", YK_DTYPE_F16, 2},  {"F64", -1, 8},
    {"I64", -1, 8},           {"U64", -1, 8},             {"I32", -1, 4},            {"U32", -1, 4},
    {"I16", -1, 2},           {"U16", -1, 2},             {"I8", -1, 1},             {"U8", -1, 1},
    {"BOOL", -1, 1},          {"F8_E4M3", -1, 1},         {"F8_E5M2", -1, 1},
};

}  // namespace

struct yk_safetensors {
    struct Entry {
        std::string name, dtype_name;
        int dtype = -1, esize = 0;
        std::vector<int64_t> shape;
        uint64_t begin = 0, end = 0;  // within the data block
    };
    int fd = -1;
    void* map = MAP_FAILED;
    size_t size = 0, data_start = 0;
    std::vector<Entry> entries;  // sorted by name
    std::map<std::string, size_t> index;

    ~yk_safetensors() {
        if (map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) ::close(fd);
    }
    const uint8_t* data(const Entry& e) const { return (const uint8_t*)map + data_start + e.begin; }
};

static yk_status st_fail(yk_safetensors* st, const std::string& msg) {
    delete st;
    yk_set_error("invalid safetensors file: " + msg);
    return YK_ERR_ARG;
}

extern "C" yk_status yk_safetensors_open(const char* path, yk_safetensors** out) {
    YK_ARG(path && out, "null argument");
    *out = nullptr;
    auto* st = new yk_safetensors();
    st->fd = ::open(path, O_RDONLY);
    if (st->fd < 0) return st_fail(st, std::string("cannot open ") + path);
    struct stat sb;
    if (fstat(st->fd, &sb) != 0) return st_fail(st, "stat failed");
    st->size = (size_t)sb.st_size;
    if (st->size < 8) return st_fail(st, "shorter than the 8-byte header length");
    st->map = mmap(nullptr, st->size, PROT_READ, MAP_PRIVATE, st->fd, 0);
    if (st->map == MAP_FAILED) return st_fail(st, "mmap failed");
    const uint8_t* b = (const uint8_t*)st->map;
    uint64_t hlen = 0;
    for (int k = 7; k >= 0; --k) hlen = (hlen << 8) | b[k];  // little-endian
    if (hlen == 0 || hlen > st->size - 8) return st_fail(st, "header length outside the file");
    st->data_start = 8 + (size_t)hlen;
    JVal root;
    if (!JParser((const char*)b + 8, (size_t)hlen).parse(root) || root.kind != JVal::OBJ)
        return st_fail(st, "header is not a JSON object");
    const uint64_t data_len = st->size - st->data_start;
    for (const auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const JVal& v = kv.second;
        if (kv.first.find('\0') != std::string::npos) return st_fail(st, "an entry name contains a NUL character");
        if (v.kind != JVal::OBJ) return st_fail(st, "entry '" + kv.first + "' is not an object");
        const JVal* dt = member(v, "dtype");
        const JVal* sh = member(v, "shape");
        const JVal* off = member(v, "data_offsets");
        if (!dt || dt->kind != JVal::STR || !sh || sh->kind != JVal::ARR || !off || off->kind != JVal::ARR ||
            off->arr.size() != 2)
            return st_fail(st, "entry '" + kv.first + "' lacks dtype / shape / data_offsets");
        yk_safetensors::Entry e;
        e.name = kv.first;
        e.dtype_name = dt->s;
        for (const auto& d : kDtypes)
            if (dt->s == d.name) {
                e.dtype = d.code;
                e.esize = d.bytes;
            }
        if (e.esize == 0) return st_fail(st, "entry '" + kv.first + "' has unknown dtype " + dt->s);
        if (sh->arr.size() > 8) return st_fail(st, "entry '" + kv.first + "' has more than 8 dimensions");
        unsigned __int128 count = 1;
        for (const auto& d : sh->arr) {
            if (d.kind != JVal::NUM || !d.is_int || d.i < 0)
                return st_fail(st, "entry '" + kv.first + "' has a bad shape");
            e.shape.push_back(d.i);
            count *= (unsigned long long)d.i;
            if (count > ((unsigned __int128)1 << 62)) return st_fail(st, "entry '" + kv.first + "' is too large");
        }
        for (const auto& o : off->arr)
            if (o.kind != JVal::NUM || !o.is_int || o.i < 0)
                return st_fail(st, "entry '" + kv.first + "' has bad data_offsets");
        e.begin = (uint64_t)off->arr[0].i;
        e.end = (uint64_t)off->arr[1].i;
        if (e.begin > e.end || e.end > data_len)
            return st_fail(st, "entry '" + kv.first + "' lies outside the data block");
        if ((unsigned __int128)(e.end - e.begin) != count * (unsigned)e.esize)
            return st_fail(st, "entry '" + kv.first + "' byte count does not match its shape");
        if (st->index.count(e.name)) return st_fail(st, "duplicate entry '" + kv.first + "'");
        st->index[e.name] = 0;
        st->entries.push_back(std::move(e));
    }
    std::sort(st->entries.begin(), st->entries.end(),
              [](const yk_safetensors::Entry& a, const yk_safetensors::Entry& b) { return a.name < b.name; });
    for (size_t i = 0; i < st->entries.size(); ++i) st->index[st->entries[i].name] = i;
    *out = st;
    return YK_OK;
}

extern "C" void yk_safetensors_close(yk_safetensors* st) { delete st; }

extern "C" int32_t yk_safetensors_count(const yk_safetensors* st) { return st ? (int32_t)st->entries.size() : 0; }

extern "C" yk_status yk_safetensors_name(const yk_safetensors* st, int32_t i, const char** name) {
    YK_ARG(st && name, "null argument");
    YK_ARG(i >= 0 && (size_t)i < st->entries.size(), "tensor index");
    *name = st->entries[(size_t)i].name.c_str();
    return YK_OK;
}

extern "C" yk_status yk_safetensors_info(const yk_safetensors* st, const char* name, yk_tensor_info* out) {
    YK_ARG(st && name && out, "null argument");
    const auto it = st->index.find(name);
    if (it == st->index.end()) {
        yk_set_error(std::string("tensor '") + name + "' not found");
        return YK_ERR_ARG;
    }
    const auto& e = st->entries[it->second];
    std::memset(out, 0, sizeof(*out));
    out->dtype = e.dtype;
    std::strncpy(out->dtype_name, e.dtype_name.c_str(), sizeof(out->dtype_name) - 1);
    out->ndim = (int32_t)e.shape.size();
    for (size_t k = 0; k < e.shape.size(); ++k) out->shape[k] = e.shape[k];
    out->data = st->data(e);
    out->nbytes = e.end - e.begin;
    return YK_OK;
}

// ---------------------------------------------------------------------------
// Device conversion
// ---------------------------------------------------------------------------
namespace yk {

__device__ __forceinline__ float load_src(const uint8_t* p, size_t i, int dt) {
    if (dt == YK_DTYPE_F32) return reinterpret_cast<const float*>(p)[i];
    if (dt == YK_DTYPE_BF16) return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(p)[i] << 16);
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
}

// A dense [nr x nc] chunk in the destination's orientation: dest row r0 + r,
// columns k0 .. k0 + nc.  v = convert(src) (+ add, when add != 0).
template <typename DT>
__global__ void load_direct_kernel(const uint8_t* __restrict__ src, int dt, int nr, int nc, DT* __restrict__ dst,
                                   size_t dst_cols, size_t row0, size_t pitch, int r0, int k0, float add) {
    const size_t n = (size_t)nr * nc;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / nc, k = i % nc;
        float v = load_src(src, i, dt);
        if (add != 0.f) v += add;  // (v + 0 would turn -0 into +0)
        dst[(row0 + (r0 + r) * pitch) * dst_cols + k0 + k] = from_f32<DT>(v);
    }
}

// A dense [nk x nr] chunk in the transposed orientation (its row i is dest
// column k0 + i): 32 x 32 tiles through shared memory, so that both the reads
// and the writes are coalesced.
template <typename DT>
__global__ void load_transpose_kernel(const uint8_t* __restrict__ src, int dt, int nk, int nr,
                                      DT* __restrict__ dst, size_t dst_cols, size_t row0, size_t pitch, int r0,
                                      int k0, float add) {
    __shared__ float tile[32][33];
    const int tk = blockIdx.y * 32, tr = blockIdx.x * 32;  // tile origin: chunk row (k), chunk column (r)
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int k = tk + y, r = tr + threadIdx.x;
        if (k < nk && r < nr) {
            const float v = load_src(src, (size_t)k * nr + r, dt);
            tile[y][threadIdx.x] = add != 0.f ? v + add : v;
        }
    }
    __syncthreads();
    for (int y = threadIdx.y; y < 32; y += blockDim.y) {
        const int r = tr + y, k = tk + threadIdx.x;
        if (k < nk && r < nr) dst[(row0 + (size_t)(r0 + r) * pitch) * dst_cols + k0 + k] = from_f32<DT>(tile[threadIdx.x][y]);
    }
}

}  // namespace yk

// ---------------------------------------------------------------------------
// Upload
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kChunkBytes = 16u << 20;  // per staging slot

size_t src_esize(int dt) { return dt == YK_DTYPE_F32 ? 4 : 2; }

// Two pinned + device staging slots and their events, for one load call.
struct Stager {
    yk_engine* e;
    void* pin[2] = {nullptr, nullptr};
    void* dev[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
    explicit Stager(yk_engine* eng) : e(eng) {}
    ~Stager() {
        cudaStreamSynchronize(e->stream);  // no copy or kernel still reads the slots
        for (int s = 0; s < 2; ++s) {
            if (ev[s]) cudaEventSynchronize(ev[s]), cudaEventDestroy(ev[s]);
            if (pin[s]) cudaFreeHost(pin[s]);
            if (dev[s]) cudaFree(dev[s]);
        }
    }
    yk_status init() {
        for (int s = 0; s < 2; ++s) {
            if (cudaMallocHost(&pin[s], kChunkBytes) != cudaSuccess || cudaMalloc(&dev[s], kChunkBytes) != cudaSuccess) {
                cudaGetLastError();
                yk_set_error("loader staging allocation failed");
                return YK_ERR_OOM;
            }
            YK_CHECK_CUDA(cudaEventCreateWithFlags(&ev[s], cudaEventDisableTiming));
        }
        return YK_OK;
    }
    // The slot's previous chunk has been converted: its buffers may be refilled.
    yk_status acquire(int s) {
        if (used[s]) YK_CHECK_CUDA(cudaEventSynchronize(ev[s]));
        return YK_OK;
    }
    yk_status submit(int s, size_t bytes) {
        YK_CHECK_CUDA(cudaMemcpyAsync(dev[s], pin[s], bytes, cudaMemcpyHostToDevice, e->stream));
        return YK_OK;
    }
    yk_status done(int s) {
        YK_CHECK_CUDA(cudaGetLastError());
        YK_CHECK_CUDA(cudaEventRecord(ev[s], e->stream));
        used[s] = true;
        return YK_OK;
    }
};

// Source of one logical tensor: the full (un-sharded) tensor as stored.
struct Source {
    const uint8_t* p;
    int dt;
    size_t rows, cols;  // stored shape
    int layout;         // YK_LAYOUT_OUT_IN: stored [out x in]; IN_OUT: stored [in x out]
    int rope_heads_hd;  // > 0: stored [out x in] rows of each head in rotate-half order (head_dim)
    float add;          // added to every element (norm gain offset)
};

// Full logical shape (out, in) of tensor t and this shard's window of it.
struct Window {
    size_t out_full, in_full, r_lo, k_lo;
};

Window window_of(const yk_model* m, int32_t t, const yk::TensorLoc& L) {
    const int tw = m->tp_world, tr = m->tp_rank;
    Window w{L.rows, L.cols, 0, 0};
    switch (t) {
        case YK_T_WQ:
        case YK_T_WK:
        case YK_T_WV:
        case YK_T_WGATE:
        case YK_T_WUP:  // column-parallel: a slice of the output rows
            w.out_full = L.rows * tw;
            w.r_lo = L.rows * tr;
            break;
        case YK_T_WO:
        case YK_T_WDOWN:  // row-parallel: a slice of the input columns
            w.in_full = L.cols * tw;
            w.k_lo = L.cols * tr;
            break;
        default: break;  // replicated
    }
    return w;
}

// Stored row of logical output row r: the inverse of the rotate-half permutation
// (a head's row 2i + j holds stored row j * head_dim / 2 + i).
inline size_t stored_row(const Source& s, size_t r) {
    if (s.rope_heads_hd <= 0) return r;
    const size_t hd = (size_t)s.rope_heads_hd, h = r / hd, w = r % hd;
    return h * hd + (w & 1) * (hd / 2) + (w >> 1);
}

template <typename DT>
yk_status upload(yk_model* m, Stager& sg, const yk::TensorLoc& L, const Window& w, const Source& s) {
    yk_engine* e = m->e;
    const size_t es = src_esize(s.dt);
    DT* dst = reinterpret_cast<DT*>(L.base);
    int slot = 0;
    if (s.layout == YK_LAYOUT_OUT_IN) {
        const size_t per = std::max<size_t>(1, kChunkBytes / (L.cols * es));
        YK_ARG(L.cols * es <= kChunkBytes, "tensor row larger than the staging slot");
        for (size_t r0 = 0; r0 < L.rows; r0 += per, slot ^= 1) {
            const size_t nr = std::min(per, L.rows - r0);
            YK_TRY(sg.acquire(slot));
            uint8_t* pin = (uint8_t*)sg.pin[slot];
            for (size_t r = 0; r < nr; ++r) {
                const size_t sr = stored_row(s, w.r_lo + r0 + r);
                std::memcpy(pin + r * L.cols * es, s.p + (sr * s.cols + w.k_lo) * es, L.cols * es);
            }
            YK_TRY(sg.submit(slot, nr * L.cols * es));
            const size_t n = nr * L.cols;
            const int blocks = (int)std::min<size_t>(148 * 8, (n + 255) / 256);
            yk::load_direct_kernel<DT><<<blocks, 256, 0, e->stream>>>((const uint8_t*)sg.dev[slot], s.dt, (int)nr,
                                                                      (int)L.cols, dst, L.cols, L.row0, L.pitch_rows,
                                                                      (int)r0, 0, s.add);
            e->launches++;
            YK_TRY(sg.done(slot));
        }
    } else {
        // stored [in x out]: stored row k is logical column k; chunks of stored rows
        const size_t per = std::min<size_t>(65535 * 32, std::max<size_t>(1, kChunkBytes / (L.rows * es)));
        YK_ARG(L.rows * es <= kChunkBytes, "tensor column larger than the staging slot");
        for (size_t k0 = 0; k0 < L.cols; k0 += per, slot ^= 1) {
            const size_t nk = std::min(per, L.cols - k0);
            YK_TRY(sg.acquire(slot));
            uint8_t* pin = (uint8_t*)sg.pin[slot];
            for (size_t k = 0; k < nk; ++k)
                std::memcpy(pin + k * L.rows * es, s.p + ((w.k_lo + k0 + k) * s.cols + w.r_lo) * es, L.rows * es);
            YK_TRY(sg.submit(slot, nk * L.rows * es));
            const dim3 grid((unsigned)((L.rows + 31) / 32), (unsigned)((nk + 31) / 32));
            yk::load_transpose_kernel<DT><<<grid, dim3(32, 8), 0, e->stream>>>(
                (const uint8_t*)sg.dev[slot], s.dt, (int)nk, (int)L.rows, dst, L.cols, L.row0, L.pitch_rows, 0,
                (int)k0, s.add);
            e->launches++;
            YK_TRY(sg.done(slot));
        }
    }
    return YK_OK;
}

yk_status load_one(yk_model* m, Stager& sg, int32_t t, int32_t layer, const Source& s) {
    YK_ARG(s.p, "null source");
    YK_ARG(s.dt == YK_DTYPE_F32 || s.dt == YK_DTYPE_BF16 || s.dt == YK_DTYPE_F16, "source dtype (F32, BF16, F16)");
    YK_ARG(s.layout == YK_LAYOUT_OUT_IN || s.layout == YK_LAYOUT_IN_OUT, "layout");
    yk::TensorLoc L;
    YK_TRY(yk::locate_tensor(m, t, layer, &L));
    const Window w = window_of(m, t, L);
    const size_t want_r = s.layout == YK_LAYOUT_OUT_IN ? w.out_full : w.in_full;
    const size_t want_c = s.layout == YK_LAYOUT_OUT_IN ? w.in_full : w.out_full;
    if (s.rows != want_r || s.cols != want_c) {
        yk_set_error("invalid argument: tensor " + std::to_string(t) + " has shape [" + std::to_string(s.rows) + " x " +
                     std::to_string(s.cols) + "], expected [" + std::to_string(want_r) + " x " +
                     std::to_string(want_c) + "]");
        return YK_ERR_ARG;
    }
    YK_ARG(L.rows <= 0x7FFFFFFF && L.cols <= 0x7FFFFFFF, "tensor extent");
    if (L.es == 2) return upload<__nv_bfloat16>(m, sg, L, w, s);
    return upload<float>(m, sg, L, w, s);
}

bool is_norm(int32_t t) { return t == YK_T_NORM1 || t == YK_T_NORM2 || t == YK_T_FINAL_NORM; }

}  // namespace

extern "C" yk_status yk_model_load_tensor(yk_model* m, int32_t tensor, int32_t layer, const void* host,
                                          int32_t src_dtype, int64_t rows, int64_t cols, int32_t layout) {
    YK_ARG(m && host, "null argument");
    YK_ARG(rows > 0 && cols > 0, "shape");
    YK_CHECK_CUDA(cudaSetDevice(m->e->device));
    Stager sg(m->e);
    YK_TRY(sg.init());
    const Source s{(const uint8_t*)host, src_dtype, (size_t)rows, (size_t)cols, layout, 0, 0.f};
    YK_TRY(load_one(m, sg, tensor, layer, s));
    YK_CHECK_CUDA(cudaStreamSynchronize(m->e->stream));
    return YK_OK;
}

// Hugging Face names of the logical tensors (Llama / Gemma layouts).
static bool hf_tensor(const std::string& name, int n_layers, int32_t* t, int32_t* layer) {
    static const std::pair<const char*, int32_t> kGlobal[] = {
        {"model.embed_tokens.weight", YK_T_EMBED}, {"model.norm.weight", YK_T_FINAL_NORM}, {"lm_head.weight", YK_T_LM_HEAD}};
    static const std::pair<const char*, int32_t> kLayer[] = {
        {"self_attn.q_proj.weight", YK_T_WQ},  {"self_attn.k_proj.weight", YK_T_WK},
        {"self_attn.v_proj.weight", YK_T_WV},  {"self_attn.o_proj.weight", YK_T_WO},
        {"mlp.gate_proj.weight", YK_T_WGATE},  {"mlp.up_proj.weight", YK_T_WUP},
        {"mlp.down_proj.weight", YK_T_WDOWN},  {"input_layernorm.weight", YK_T_NORM1},
        {"post_attention_layernorm.weight", YK_T_NORM2}};
    for (const auto& g : kGlobal)
        if (name == g.first) {
            *t = g.second;
            *layer = 0;
            return true;
        }
    const std::string pre = "model.layers.";
    if (name.compare(0, pre.size(), pre) != 0) return false;
    size_t p = pre.size(), q = p;
    while (q < name.size() && name[q] >= '0' && name[q] <= '9') ++q;
    // canonical decimal only ("7", not "07"), so that one name maps to each slot
    if (q == p || q - p > 6 || (name[p] == '0' && q - p > 1) || q >= name.size() || name[q] != '.') return false;
    const int l = std::atoi(name.substr(p, q - p).c_str());
    if (l >= n_layers) return false;
    const std::string rest = name.substr(q + 1);
    for (const auto& e : kLayer)
        if (rest == e.first) {
            *t = e.second;
            *layer = l;
            return true;
        }
    return false;
}

extern "C" yk_status yk_hf_tensor_id(const char* name, int32_t n_layers, int32_t* tensor, int32_t* layer) {
    YK_ARG(name && tensor && layer && n_layers > 0, "null argument");
    if (!hf_tensor(name, n_layers, tensor, layer)) {
        yk_set_error(std::string("'") + name + "' is not a weight of this module's layout");
        return YK_ERR_ARG;
    }
    return YK_OK;
}

extern "C" yk_status yk_model_load_safetensors(yk_model* m, yk_safetensors* const* files, int32_t n_files,
                                               float norm_offset, int32_t flags, int32_t* n_loaded) {
    YK_ARG(m && files && n_files > 0, "null argument");
    YK_ARG((flags & ~YK_LOAD_ROPE_HALF) == 0, "flags");
    if (n_loaded) *n_loaded = 0;
    const auto& c = m->cfg;
    const int L = c.n_layers;
    // every (tensor, layer) slot: which file holds it
    std::vector<std::pair<const yk_safetensors*, const yk_safetensors::Entry*>> slot((size_t)(3 + 9 * L),
                                                                                     {nullptr, nullptr});
    auto slot_of = [&](int32_t t, int32_t l) -> size_t {
        if (t == YK_T_EMBED) return 0;
        if (t == YK_T_FINAL_NORM) return 1;
        if (t == YK_T_LM_HEAD) return 2;
        return 3 + (size_t)l * 9 + (size_t)(t - YK_T_WQ);
    };
    for (int f = 0; f < n_files; ++f) {
        YK_ARG(files[f], "null file handle");
        for (const auto& e : files[f]->entries) {
            int32_t t, l;
            if (!hf_tensor(e.name, L, &t, &l)) {
                // buffers that are not weights of this module's layers are skipped;
                // an unknown tensor of a decoder layer is a layer this module lacks
                if (e.name.compare(0, 13, "model.layers.") == 0 && e.name.find("rotary_emb") == std::string::npos) {
                    yk_set_error("unsupported checkpoint tensor '" + e.name + "'");
                    return YK_ERR_UNSUPPORTED;
                }
                continue;
            }
            auto& s = slot[slot_of(t, l)];
            if (s.first) {
                yk_set_error("tensor '" + e.name + "' appears in more than one file");
                return YK_ERR_ARG;
            }
            s = {files[f], &e};
        }
    }
    if (!slot[2].first) slot[2] = slot[0];  // tied embeddings: the LM head is the embedding table
    YK_CHECK_CUDA(cudaSetDevice(m->e->device));
    Stager sg(m->e);
    YK_TRY(sg.init());
    int32_t loaded = 0;
    for (int32_t t = 0; t <= YK_T_LM_HEAD; ++t) {
        const bool per_layer = t >= YK_T_WQ && t <= YK_T_NORM2;
        for (int32_t l = 0; l < (per_layer ? L : 1); ++l) {
            const auto& s = slot[slot_of(t, l)];
            if (!s.first) {
                yk_set_error("checkpoint lacks tensor " + std::to_string(t) + (per_layer ? " of layer " + std::to_string(l) : ""));
                return YK_ERR_ARG;
            }
            const auto& e = *s.second;
            if (e.dtype < 0) {
                yk_set_error("tensor '" + e.name + "' has dtype " + e.dtype_name + " (F32, BF16 or F16 only)");
                return YK_ERR_UNSUPPORTED;
            }
            Source src{s.first->data(e), e.dtype, 0, 0, YK_LAYOUT_OUT_IN, 0, 0.f};
            if (e.shape.size() == 1) {
                src.rows = 1;
                src.cols = (size_t)e.shape[0];
            } else if (e.shape.size() == 2) {
                src.rows = (size_t)e.shape[0];
                src.cols = (size_t)e.shape[1];
            } else {
                yk_set_error("tensor '" + e.name + "' is not a matrix or a vector");
                return YK_ERR_ARG;
            }
            if ((flags & YK_LOAD_ROPE_HALF) && (t == YK_T_WQ || t == YK_T_WK)) src.rope_heads_hd = c.head_dim;
            if (is_norm(t)) src.add = norm_offset;
            const yk_status st = load_one(m, sg, t, l, src);
            if (st != YK_OK) {
                yk_set_error("loading '" + e.name + "': " + [] {
                    char buf[512];
                    yk_last_error(buf, sizeof buf);
                    return std::string(buf);
                }());
                return st;
            }
            ++loaded;
        }
    }
    YK_CHECK_CUDA(cudaStreamSynchronize(m->e->stream));
    if (n_loaded) *n_loaded = loaded;
    return YK_OK;
}
