#include "gguf.h"

#include <cstdio>
#include <cstring>
#include <memory>

namespace mcpm {

uint64_t ggml_nbytes(uint32_t type, uint64_t n) {
    switch (type) {
        case 0: return n * 4;                                  // F32
        case 1: return n * 2;                                  // F16
        case 8: return n % 32 ? 0 : n / 32 * 34;               // Q8_0
        case 12: return n % 256 ? 0 : n / 256 * 144;          // Q4_K
        case 14: return n % 256 ? 0 : n / 256 * 210;          // Q6_K
        default: return 0;
    }
}

namespace {

struct Reader {
    FILE* f;
    bool ok = true;
    template <typename T>
    T get() {
        T v{};
        if (ok && std::fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1ull << 30)) {
            ok = false;
            return {};
        }
        std::string s(n, '\0');
        if (n && std::fread(&s[0], 1, n, f) != n) ok = false;
        return s;
    }
    void skip(uint64_t n) {
        if (ok && std::fseek(f, static_cast<long>(n), SEEK_CUR) != 0) ok = false;
    }
};

// GGUF value types: 0 u8, 1 i8, 2 u16, 3 i16, 4 u32, 5 i32, 6 f32, 7 bool, 8 str, 9 arr,
// 10 u64, 11 i64, 12 f64.
int scalar_size(uint32_t t) {
    switch (t) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: return 0;
    }
}

bool read_value(Reader& r, uint32_t t, const std::string& key, GGUFFile& out) {
    switch (t) {
        case 0: out.u64_kv[key] = r.get<uint8_t>(); return r.ok;
        case 1: out.u64_kv[key] = static_cast<uint64_t>(r.get<int8_t>()); return r.ok;
        case 2: out.u64_kv[key] = r.get<uint16_t>(); return r.ok;
        case 3: out.u64_kv[key] = static_cast<uint64_t>(r.get<int16_t>()); return r.ok;
        case 4: out.u64_kv[key] = r.get<uint32_t>(); return r.ok;
        case 5: out.u64_kv[key] = static_cast<uint64_t>(r.get<int32_t>()); return r.ok;
        case 6: out.f_kv[key] = r.get<float>(); return r.ok;
        case 7: out.u64_kv[key] = r.get<uint8_t>(); return r.ok;
        case 8: r.str(); return r.ok;
        case 10: out.u64_kv[key] = r.get<uint64_t>(); return r.ok;
        case 11: out.u64_kv[key] = static_cast<uint64_t>(r.get<int64_t>()); return r.ok;
        case 12: out.f_kv[key] = r.get<double>(); return r.ok;
        case 9: {
            const uint32_t et = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            if (!r.ok) return false;
            if (et == 8) {
                for (uint64_t i = 0; i < n && r.ok; ++i) r.str();
            } else if (scalar_size(et)) {
                r.skip(n * scalar_size(et));
            } else {
                return false;   // nested arrays are not used by this model family
            }
            return r.ok;
        }
        default: return false;
    }
}

}  // namespace

std::string gguf_read(const std::string& path, GGUFFile& out) {
    std::unique_ptr<FILE, int (*)(FILE*)> fp(std::fopen(path.c_str(), "rb"), &std::fclose);
    if (!fp) return "cannot open " + path;
    std::fseek(fp.get(), 0, SEEK_END);
    out.file_size = static_cast<uint64_t>(std::ftell(fp.get()));
    std::fseek(fp.get(), 0, SEEK_SET);
    Reader r{fp.get()};
    char magic[4];
    if (std::fread(magic, 1, 4, fp.get()) != 4 || std::memcmp(magic, "GGUF", 4) != 0) return "not a GGUF file";
    const uint32_t version = r.get<uint32_t>();
    if (!r.ok || (version != 2 && version != 3)) return "unsupported GGUF version";
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > 100000 || n_kv > 100000) return "implausible GGUF header counts";
    for (uint64_t i = 0; i < n_kv; ++i) {
        const std::string key = r.str();
        const uint32_t t = r.get<uint32_t>();
        if (!r.ok || !read_value(r, t, key, out)) return "truncated or malformed GGUF metadata";
    }
    auto it = out.u64_kv.find("general.alignment");
    if (it != out.u64_kv.end()) out.alignment = static_cast<uint32_t>(it->second);
    if (out.alignment == 0 || (out.alignment & (out.alignment - 1))) return "bad GGUF alignment";
    std::vector<GGUFTensor> ts(n_tensors);
    for (auto& t : ts) {
        t.name = r.str();
        const uint32_t nd = r.get<uint32_t>();
        if (!r.ok || nd == 0 || nd > 4) return "malformed tensor info";
        uint64_t n = 1;
        for (uint32_t d = 0; d < nd; ++d) {
            t.dims.push_back(r.get<uint64_t>());
            n *= t.dims.back();
        }
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        if (!r.ok) return "truncated tensor info";
        t.nbytes = ggml_nbytes(t.type, n);
    }
    const uint64_t hdr_end = static_cast<uint64_t>(std::ftell(fp.get()));
    out.data_start = (hdr_end + out.alignment - 1) / out.alignment * out.alignment;
    for (auto& t : ts) {
        t.offset += out.data_start;
        if (t.nbytes && t.offset + t.nbytes > out.file_size) return "tensor " + t.name + " extends past end of file";
    }
    out.tensors = std::move(ts);
    return {};
}

}  // namespace mcpm
