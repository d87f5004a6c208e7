// gx_gguf.cpp — routed-expert layers straight from a GGUF model file into the HBM arena
// (gx_gguf_inspect_layer, gx_upload_layer_gguf). It takes the place, for this path, of the Zig host's
// GGUF reader (src/gguf.zig), tensor binding (src/model.zig:395-421: the stacked expert tensors,
// the router, the shared expert, the prism.hadamard sign lookup of :305-330) and expert-arena
// setup (src/gpu_engine.zig:593-668). Host code only: the file is parsed from a bounded header
// prefix, the tensors the layer needs are read with pread and handed to gx_upload_layer /
// gx_upload_shared, which own the device side.
//
// Header rules follow the reference parser (src/gguf.zig:263-334): magic "GGUF", version 3,
// at most 10^6 tensors and metadata entries, unique non-empty keys, value types 0..12, arrays
// nested at most 8 deep with at most 2^24 elements, booleans 0 or 1, general.alignment a power
// of two up to 65536 (32 if absent), unique tensor names, rank 1..4, non-zero dimensions,
// aligned tensor offsets, tensor byte lengths from each type's block size, every tensor inside
// the file and no two overlapping.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/gyro_moe.h"
#include "gx_tile.h"

namespace {

constexpr uint64_t kMaxHeaderBytes = 64ull << 20;

bool gguf_debug() {
    const char *v = std::getenv("GX_DEBUG");
    return v && v[0] && v[0] != '0';
}

gx_result reject(gx_result code, const char *why) {
    if (gguf_debug()) std::fprintf(stderr, "gyro_moe: GGUF: %s\n", why);
    return code;
}

enum VType : uint32_t {
    V_U8 = 0, V_I8, V_U16, V_I16, V_U32, V_I32, V_F32, V_BOOL, V_STR, V_ARR, V_U64, V_I64, V_F64
};

struct Entry {
    uint32_t kind = 0;
    const uint8_t *raw = nullptr;   // the value's bytes inside the header prefix
    size_t len = 0;
};

struct Tensor {
    uint32_t rank = 0, type = 0;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t rel = 0, off = 0, bytes = 0;
    bool sized = false;
};

// Bounds-checked little-endian reader over the header prefix.
struct Cursor {
    const uint8_t *p;
    size_t n, pos = 0;
    bool ok = true;
    bool take(size_t k, const uint8_t **out) {
        if (!ok || k > n - pos) return ok = false;
        *out = p + pos;
        pos += k;
        return true;
    }
    template <typename T>
    T num() {
        const uint8_t *b = nullptr;
        T v{};
        if (take(sizeof(T), &b)) std::memcpy(&v, b, sizeof(T));
        return v;
    }
    bool str(std::string *out) {
        const uint64_t len = num<uint64_t>();
        const uint8_t *b = nullptr;
        if (!ok || len > kMaxHeaderBytes || !take((size_t)len, &b)) return ok = false;
        if (out) out->assign(reinterpret_cast<const char *>(b), (size_t)len);
        return true;
    }
    bool skip(uint32_t kind, int depth) {
        if (depth > 8) return ok = false;
        const uint8_t *b = nullptr;
        switch (kind) {
            case V_U8: case V_I8: return take(1, &b);
            case V_BOOL: return take(1, &b) && (*b <= 1 || (ok = false));
            case V_U16: case V_I16: return take(2, &b);
            case V_U32: case V_I32: case V_F32: return take(4, &b);
            case V_U64: case V_I64: case V_F64: return take(8, &b);
            case V_STR: return str(nullptr);
            case V_ARR: {
                const uint32_t elem = num<uint32_t>();
                const uint64_t count = num<uint64_t>();
                if (!ok || elem > V_F64 || count > (16u << 20)) return ok = false;
                for (uint64_t i = 0; i < count && ok; ++i) skip(elem, depth + 1);
                return ok;
            }
            default: return ok = false;
        }
    }
};

// Block size in weights and bytes of the tensor types a layer can carry (src/gguf.zig:126-137).
bool type_layout(uint32_t t, uint64_t *weights, uint64_t *bytes) {
    if (gx::type_k(t)) { *weights = 128; *bytes = (uint64_t)gx::type_block_bytes(t); return true; }
    switch (t) {
        case 0: *weights = 1; *bytes = 4; return true;    // F32
        case 1: *weights = 1; *bytes = 2; return true;    // F16
        case 8: *weights = 32; *bytes = 34; return true;  // Q8_0
        case 30: *weights = 1; *bytes = 2; return true;   // BF16
        default: return false;
    }
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t *out) {
    if (a && b > UINT64_MAX / a) return false;
    *out = a * b;
    return true;
}

struct File {
    int fd = -1;
    uint64_t size = 0;
    std::vector<uint8_t> head;
    std::map<std::string, Entry> meta;
    std::map<std::string, Tensor> tensors;
    ~File() {
        if (fd >= 0) close(fd);
    }

    bool read_at(uint64_t off, void *dst, uint64_t bytes) const {
        uint8_t *p = static_cast<uint8_t *>(dst);
        while (bytes) {
            const ssize_t got = pread(fd, p, (size_t)std::min<uint64_t>(bytes, 1u << 30), (off_t)off);
            if (got <= 0) return false;
            p += got;
            off += (uint64_t)got;
            bytes -= (uint64_t)got;
        }
        return true;
    }

    gx_result open_parse(const char *path) {
        fd = open(path, O_RDONLY | O_CLOEXEC);
        if (fd < 0) return reject(GX_E_INVALIDARG, "cannot open the file");
        struct stat st {};
        if (fstat(fd, &st) != 0) return reject(GX_E_INVALIDARG, "cannot stat the file");
        size = (uint64_t)st.st_size;
        head.resize((size_t)std::min<uint64_t>(size, kMaxHeaderBytes));
        if (!read_at(0, head.data(), head.size())) return reject(GX_E_INVALIDARG, "cannot read the header");
        Cursor c{head.data(), head.size()};
        const uint8_t *magic = nullptr;
        if (!c.take(4, &magic) || std::memcmp(magic, "GGUF", 4) != 0) return reject(GX_E_INVALIDARG, "bad magic");
        if (c.num<uint32_t>() != 3) return reject(GX_E_UNSUPPORTED, "only GGUF version 3");
        const uint64_t n_tensors = c.num<uint64_t>(), n_meta = c.num<uint64_t>();
        if (!c.ok || n_tensors > 1000000 || n_meta > 1000000) return reject(GX_E_INVALIDARG, "entry counts");
        uint64_t alignment = 32;
        for (uint64_t i = 0; i < n_meta; ++i) {
            std::string key;
            if (!c.str(&key) || key.empty() || key.size() > 65535) return reject(GX_E_INVALIDARG, "metadata key");
            Entry e;
            e.kind = c.num<uint32_t>();
            const size_t start = c.pos;
            if (!c.ok || !c.skip(e.kind, 0)) return reject(GX_E_INVALIDARG, "metadata value");
            e.raw = head.data() + start;
            e.len = c.pos - start;
            if (!meta.emplace(key, e).second) return reject(GX_E_INVALIDARG, "duplicate metadata key");
            if (key == "general.alignment") {
                if (e.kind != V_U32) return reject(GX_E_INVALIDARG, "general.alignment is not uint32");
                uint32_t v;
                std::memcpy(&v, e.raw, 4);
                alignment = v;
            }
        }
        if (alignment == 0 || alignment > 65536 || (alignment & (alignment - 1)))
            return reject(GX_E_INVALIDARG, "alignment");
        for (uint64_t i = 0; i < n_tensors; ++i) {
            std::string name;
            if (!c.str(&name) || name.empty() || name.size() > 4096) return reject(GX_E_INVALIDARG, "tensor name");
            Tensor t;
            t.rank = c.num<uint32_t>();
            if (!c.ok || t.rank == 0 || t.rank > 4) return reject(GX_E_INVALIDARG, "tensor rank");
            for (uint32_t d = 0; d < t.rank; ++d) {
                t.dims[d] = c.num<uint64_t>();
                if (t.dims[d] == 0) return reject(GX_E_INVALIDARG, "zero dimension");
            }
            t.type = c.num<uint32_t>();
            t.rel = c.num<uint64_t>();
            if (!c.ok) return reject(GX_E_INVALIDARG, "truncated tensor info");
            if (t.rel % alignment) return reject(GX_E_INVALIDARG, "misaligned tensor offset");
            uint64_t bw, bb;
            if (type_layout(t.type, &bw, &bb)) {
                if (t.dims[0] % bw) return reject(GX_E_INVALIDARG, "row is not a whole number of blocks");
                uint64_t n = 0;
                if (!mul_ok(t.dims[0] / bw, bb, &n)) return reject(GX_E_INVALIDARG, "tensor size overflow");
                for (uint32_t d = 1; d < t.rank; ++d)
                    if (!mul_ok(n, t.dims[d], &n)) return reject(GX_E_INVALIDARG, "tensor size overflow");
                t.bytes = n;
                t.sized = true;
            }
            if (!tensors.emplace(name, t).second) return reject(GX_E_INVALIDARG, "duplicate tensor name");
        }
        const uint64_t data = (c.pos + alignment - 1) & ~(alignment - 1);
        if (data > size) return reject(GX_E_INVALIDARG, "data section past the end of the file");
        std::vector<Tensor *> order;
        for (auto &kv : tensors) {
            Tensor &t = kv.second;
            t.off = data + t.rel;
            if (t.off < data || t.off >= size) return reject(GX_E_INVALIDARG, "tensor outside the file");
            if (t.sized && (t.bytes > size || t.off > size - t.bytes)) return reject(GX_E_INVALIDARG, "tensor outside the file");
            order.push_back(&t);
        }
        std::sort(order.begin(), order.end(), [](const Tensor *a, const Tensor *b) { return a->off < b->off; });
        for (size_t i = 0; i + 1 < order.size(); ++i) {
            if (order[i + 1]->off == order[i]->off) return reject(GX_E_INVALIDARG, "overlapping tensors");
            if (order[i]->sized && order[i]->off + order[i]->bytes > order[i + 1]->off)
                return reject(GX_E_INVALIDARG, "overlapping tensors");
        }
        return GX_OK;
    }

    const Entry *get(const std::string &key) const {
        auto it = meta.find(key);
        return it == meta.end() ? nullptr : &it->second;
    }
    const Tensor *tensor(const std::string &name) const {
        auto it = tensors.find(name);
        return it == tensors.end() ? nullptr : &it->second;
    }
    bool text(const std::string &key, std::string *out) const {
        const Entry *e = get(key);
        if (!e || e->kind != V_STR) return false;
        Cursor c{e->raw, e->len};
        return c.str(out);
    }
    bool unsigned_value(const std::string &key, uint64_t *out) const {
        const Entry *e = get(key);
        if (!e) return false;
        Cursor c{e->raw, e->len};
        switch (e->kind) {
            case V_U8: *out = c.num<uint8_t>(); return c.ok;
            case V_U16: *out = c.num<uint16_t>(); return c.ok;
            case V_U32: *out = c.num<uint32_t>(); return c.ok;
            case V_U64: *out = c.num<uint64_t>(); return c.ok;
            default: return false;
        }
    }
    bool float_value(const std::string &key, float *out) const {
        const Entry *e = get(key);
        if (!e) return false;
        Cursor c{e->raw, e->len};
        if (e->kind == V_F32) { *out = c.num<float>(); return c.ok; }
        if (e->kind == V_F64) { *out = (float)c.num<double>(); return c.ok; }
        return false;
    }
    bool strings(const std::string &key, std::vector<std::string> *out) const {
        const Entry *e = get(key);
        if (!e || e->kind != V_ARR) return false;
        Cursor c{e->raw, e->len};
        if (c.num<uint32_t>() != V_STR) return false;
        const uint64_t n = c.num<uint64_t>();
        out->resize((size_t)n);
        for (auto &s : *out)
            if (!c.str(&s)) return false;
        return c.ok;
    }
    bool ints32(const std::string &key, std::vector<int32_t> *out) const {
        const Entry *e = get(key);
        if (!e || e->kind != V_ARR) return false;
        Cursor c{e->raw, e->len};
        if (c.num<uint32_t>() != V_I32) return false;
        const uint64_t n = c.num<uint64_t>();
        out->resize((size_t)n);
        for (auto &v : *out) v = c.num<int32_t>();
        return c.ok;
    }
};

std::string blk(uint32_t layer, const char *suffix) { return "blk." + std::to_string(layer) + "." + suffix; }

// The layer's bindings (src/model.zig:408-421) and hyper-parameters.
struct LayerPlan {
    const Tensor *gate = nullptr, *up = nullptr, *down = nullptr, *router = nullptr;
    const Tensor *sh_gate = nullptr, *sh_up = nullptr, *sh_down = nullptr, *sh_inp = nullptr;
    gx_gguf_layer_info info{};
    std::vector<float> gate_signs, down_signs;
};

// Signs of a listed tensor: the sign vector whose width is the tensor's input width
// (src/model.zig:305-330), or none when the tensor is not listed. Validation as
// src/gguf.zig:192-252 for the explicit mode the reference model uses.
gx_result signs_of(const File &f, const std::string &name, uint64_t width, std::vector<float> *out) {
    out->clear();
    std::vector<std::string> names;
    if (!f.strings("prism.hadamard.weight_names", &names)) return GX_OK;  // nothing rotated
    if (std::find(names.begin(), names.end(), name) == names.end()) return GX_OK;
    uint64_t v = 0;
    if (!f.unsigned_value("prism.hadamard.version", &v) || v != 1) return reject(GX_E_UNSUPPORTED, "prism.hadamard.version");
    if (!f.unsigned_value("prism.hadamard.block_size", &v) || v != 128)
        return reject(GX_E_UNSUPPORTED, "prism.hadamard.block_size must be 128");
    std::string s;
    if (!f.text("prism.hadamard.transform", &s) || s != "normalized-sylvester-walsh-hadamard")
        return reject(GX_E_UNSUPPORTED, "prism.hadamard.transform");
    if (!f.text("prism.hadamard.axis", &s) || s != "input-last-dimension") return reject(GX_E_UNSUPPORTED, "prism.hadamard.axis");
    if (!f.text("prism.hadamard.sign_mode", &s)) return reject(GX_E_INVALIDARG, "prism.hadamard.sign_mode");
    if (s == "identity") {
        out->assign((size_t)width, 1.0f);
        return GX_OK;
    }
    if (s != "explicit") return reject(GX_E_UNSUPPORTED, "prism.hadamard.sign_mode");
    std::vector<int32_t> widths, values;
    if (!f.ints32("prism.hadamard.sign_widths", &widths) || !f.ints32("prism.hadamard.sign_values", &values))
        return reject(GX_E_INVALIDARG, "prism.hadamard sign arrays");
    uint64_t off = 0, sum = 0;
    bool found = false;
    for (size_t i = 0; i < widths.size(); ++i) {
        if (widths[i] <= 0 || widths[i] % 128) return reject(GX_E_INVALIDARG, "prism.hadamard.sign_widths");
        for (size_t j = 0; j < i; ++j)
            if (widths[j] == widths[i]) return reject(GX_E_INVALIDARG, "repeated sign width");
        if (!found && (uint64_t)widths[i] == width) {
            found = true;
            off = sum;
        }
        sum += (uint64_t)widths[i];
    }
    if (values.size() != sum) return reject(GX_E_INVALIDARG, "prism.hadamard.sign_values length");
    if (!found) return reject(GX_E_INVALIDARG, "no sign vector of the tensor's width");
    out->resize((size_t)width);
    for (uint64_t i = 0; i < width; ++i) {
        const int32_t sv = values[(size_t)(off + i)];
        if (sv != 1 && sv != -1) return reject(GX_E_INVALIDARG, "sign value not +-1");
        (*out)[(size_t)i] = (float)sv;
    }
    return GX_OK;
}

gx_result plan_layer(const File &f, uint32_t layer, LayerPlan *p) {
    p->gate = f.tensor(blk(layer, "ffn_gate_exps.weight"));
    p->up = f.tensor(blk(layer, "ffn_up_exps.weight"));
    p->down = f.tensor(blk(layer, "ffn_down_exps.weight"));
    p->router = f.tensor(blk(layer, "ffn_gate_inp.weight"));
    if (!p->gate || !p->up || !p->down || !p->router) return reject(GX_E_INVALIDARG, "missing routed-expert tensor");
    const Tensor &g = *p->gate;
    if (g.rank != 3 || p->up->rank != 3 || p->down->rank != 3) return reject(GX_E_INVALIDARG, "expert tensors are not 3-D");
    const uint64_t E = g.dims[0], F = g.dims[1], NE = g.dims[2];
    if (p->up->dims[0] != E || p->up->dims[1] != F || p->up->dims[2] != NE || p->down->dims[0] != F ||
        p->down->dims[1] != E || p->down->dims[2] != NE)
        return reject(GX_E_INVALIDARG, "expert tensor shapes disagree");
    if (!gx::type_k(g.type) || p->up->type != g.type || p->down->type != g.type)
        return reject(GX_E_UNSUPPORTED, "expert tensors must share one Gyro type");
    const Tensor &r = *p->router;
    if (r.rank != 2 || r.dims[0] != E || r.dims[1] != NE) return reject(GX_E_INVALIDARG, "router shape");
    if (r.type != 0 && r.type != 1 && r.type != 30) return reject(GX_E_UNSUPPORTED, "router type");
    std::string arch;
    if (!f.text("general.architecture", &arch)) return reject(GX_E_INVALIDARG, "general.architecture");
    uint64_t used = 0;
    if (!f.unsigned_value(arch + ".expert_used_count", &used)) return reject(GX_E_INVALIDARG, "expert_used_count");
    uint64_t count = 0;
    if (f.unsigned_value(arch + ".expert_count", &count) && count != NE) return reject(GX_E_INVALIDARG, "expert_count");
    float scale = 0.f;
    if (f.get(arch + ".expert_weights_scale") && !f.float_value(arch + ".expert_weights_scale", &scale))
        return reject(GX_E_INVALIDARG, "expert_weights_scale");
    gx_gguf_layer_info &in = p->info;
    in.type_id = g.type;
    in.n_expert = (uint32_t)NE;
    in.n_embd = (uint32_t)E;
    in.n_ff = (uint32_t)F;
    in.n_used = (uint32_t)used;
    in.expert_weights_scale = scale;
    in.shared_type = GX_SHARED_NONE;
    gx_result rs = signs_of(f, blk(layer, "ffn_gate_exps.weight"), E, &p->gate_signs);
    if (rs != GX_OK) return rs;
    std::vector<float> up_signs;
    rs = signs_of(f, blk(layer, "ffn_up_exps.weight"), E, &up_signs);
    if (rs != GX_OK) return rs;
    if (up_signs != p->gate_signs) return reject(GX_E_INVALIDARG, "gate and up must share their signs");
    rs = signs_of(f, blk(layer, "ffn_down_exps.weight"), F, &p->down_signs);
    if (rs != GX_OK) return rs;
    in.rotated = (p->gate_signs.empty() ? 0u : 1u) | (p->down_signs.empty() ? 0u : 2u);
    p->sh_gate = f.tensor(blk(layer, "ffn_gate_shexp.weight"));
    p->sh_up = f.tensor(blk(layer, "ffn_up_shexp.weight"));
    p->sh_down = f.tensor(blk(layer, "ffn_down_shexp.weight"));
    p->sh_inp = f.tensor(blk(layer, "ffn_gate_inp_shexp.weight"));
    const int present = !!p->sh_gate + !!p->sh_up + !!p->sh_down + !!p->sh_inp;
    if (present != 0 && present != 4) return reject(GX_E_INVALIDARG, "incomplete shared expert");
    if (present == 4) {
        const Tensor &sg = *p->sh_gate;
        const uint64_t SF = sg.dims[1];
        if (sg.rank != 2 || sg.dims[0] != E || p->sh_up->rank != 2 || p->sh_up->dims[0] != E || p->sh_up->dims[1] != SF ||
            p->sh_down->rank != 2 || p->sh_down->dims[0] != SF || p->sh_down->dims[1] != E)
            return reject(GX_E_INVALIDARG, "shared-expert shapes");
        if (p->sh_up->type != sg.type || p->sh_down->type != sg.type) return reject(GX_E_UNSUPPORTED, "shared-expert types differ");
        const Tensor &si = *p->sh_inp;
        if (si.type != 0 || si.dims[0] * si.dims[1] * si.dims[2] * si.dims[3] != E)
            return reject(GX_E_INVALIDARG, "shared-expert gate");
        in.shared_type = sg.type;
        in.shared_ff = (uint32_t)SF;
    }
    return GX_OK;
}

bool read_tensor(const File &f, const Tensor &t, std::vector<uint8_t> *out) {
    if (!t.sized) return false;
    out->resize((size_t)t.bytes);
    return f.read_at(t.off, out->data(), t.bytes);
}

// Router rows as f32 (f16 and bf16 widen exactly).
bool router_f32(const File &f, const Tensor &t, std::vector<float> *out) {
    std::vector<uint8_t> raw;
    if (!read_tensor(f, t, &raw)) return false;
    const size_t n = (size_t)(t.dims[0] * t.dims[1]);
    out->resize(n);
    if (t.type == 0) {
        std::memcpy(out->data(), raw.data(), n * 4);
        return true;
    }
    for (size_t i = 0; i < n; ++i) {
        const uint16_t h = (uint16_t)(raw[2 * i] | (raw[2 * i + 1] << 8));
        uint32_t bits;
        if (t.type == 30) {
            bits = (uint32_t)h << 16;
        } else {  // binary16 -> binary32, subnormals included
            const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u;
            uint32_t m = h & 1023u;
            if (e == 31) bits = sign | 0x7f800000u | (m << 13);
            else if (e) bits = sign | ((e + 112u) << 23) | (m << 13);
            else if (!m) bits = sign;
            else {
                uint32_t oe = 113;
                while (!(m & 1024u)) { m <<= 1; --oe; }
                bits = sign | (oe << 23) | ((m & 1023u) << 13);
            }
        }
        std::memcpy(&(*out)[i], &bits, 4);
    }
    return true;
}

}  // namespace

extern "C" {

GX_API gx_result gx_gguf_inspect_layer(const char *path, uint32_t gguf_layer, gx_gguf_layer_info *out) {
    if (!path || !out) return GX_E_INVALIDARG;
    File f;
    gx_result r = f.open_parse(path);
    if (r != GX_OK) return r;
    LayerPlan p;
    r = plan_layer(f, gguf_layer, &p);
    if (r != GX_OK) return r;
    *out = p.info;
    return GX_OK;
}

GX_API gx_result gx_upload_layer_gguf(gx_context *context, uint32_t layer, const char *path, uint32_t gguf_layer,
                                      uint32_t timeout_ms) {
    if (!context || !path) return GX_E_INVALIDARG;
    File f;
    gx_result r = f.open_parse(path);
    if (r != GX_OK) return r;
    LayerPlan p;
    r = plan_layer(f, gguf_layer, &p);
    if (r != GX_OK) return r;
    std::vector<uint8_t> gate, up, down;
    std::vector<float> router;
    if (!read_tensor(f, *p.gate, &gate) || !read_tensor(f, *p.up, &up) || !read_tensor(f, *p.down, &down) ||
        !router_f32(f, *p.router, &router))
        return reject(GX_E_INVALIDARG, "cannot read a routed-expert tensor");
    gx_layer_desc d{};
    d.type_id = p.info.type_id;
    d.n_expert = p.info.n_expert;
    d.n_embd = p.info.n_embd;
    d.n_ff = p.info.n_ff;
    d.n_used = p.info.n_used;
    d.expert_weights_scale = p.info.expert_weights_scale;
    d.gate = gate.data();
    d.up = up.data();
    d.down = down.data();
    d.gate_bytes = gate.size();
    d.up_bytes = up.size();
    d.down_bytes = down.size();
    d.router = router.data();
    d.gate_signs = p.gate_signs.empty() ? nullptr : p.gate_signs.data();
    d.up_signs = d.gate_signs;
    d.down_signs = p.down_signs.empty() ? nullptr : p.down_signs.data();
    r = gx_upload_layer(context, layer, &d, timeout_ms);
    if (r != GX_OK || p.info.shared_type == GX_SHARED_NONE) return r;
    std::vector<uint8_t> sg, su, sd, si;
    if (!read_tensor(f, *p.sh_gate, &sg) || !read_tensor(f, *p.sh_up, &su) || !read_tensor(f, *p.sh_down, &sd) ||
        !read_tensor(f, *p.sh_inp, &si))
        return reject(GX_E_INVALIDARG, "cannot read a shared-expert tensor");
    gx_shared_desc s{};
    s.type_id = p.info.shared_type;
    s.n_ff = p.info.shared_ff;
    s.gate = sg.data();
    s.up = su.data();
    s.down = sd.data();
    s.gate_bytes = sg.size();
    s.up_bytes = su.size();
    s.down_bytes = sd.size();
    s.gate_inp = reinterpret_cast<const float *>(si.data());
    return gx_upload_shared(context, layer, &s, timeout_ms);
}

}  // extern "C"
