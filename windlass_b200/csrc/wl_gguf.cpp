// GGUF reader: the header and tensor-index rules of GgufModelFile.ReadHeader (src/Gguf.cs:143-208).
#include "wl_gguf.h"
#include "wl_common.h"
#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace wl {

namespace {
struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    const std::string& path;
    void need(size_t n)
    {
        if ((size_t)(end - p) < n) WL_THROW(WL_EFORMAT, path + ": unexpected end of GGUF header.");
    }
    template <typename T> T get()
    {
        need(sizeof(T));
        T v;
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str()
    {
        const uint64_t n = get<uint64_t>();
        if (n > (uint64_t)(end - p)) WL_THROW(WL_EFORMAT, path + ": GGUF string too long.");
        std::string s((const char*)p, (size_t)n);
        p += n;
        return s;
    }
};

int scalar_size(int t)
{
    switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    }
    return -1;
}

void read_scalar(Reader& r, int t, GgufValue& v)
{
    switch (t) {
    case 0: v.i = r.get<uint8_t>(); break;
    case 1: v.i = r.get<int8_t>(); break;
    case 2: v.i = r.get<uint16_t>(); break;
    case 3: v.i = r.get<int16_t>(); break;
    case 4: v.i = r.get<uint32_t>(); break;
    case 5: v.i = r.get<int32_t>(); break;
    case 6: v.f = r.get<float>(); v.i = (int64_t)v.f; return;
    case 7: v.i = r.get<uint8_t>() != 0; break;
    case 8: v.s = r.str(); return;
    case 10: v.i = (int64_t)r.get<uint64_t>(); break;
    case 11: v.i = r.get<int64_t>(); break;
    case 12: v.f = r.get<double>(); v.i = (int64_t)v.f; return;
    default: WL_THROW(WL_EFORMAT, r.path + ": unknown GGUF value type " + std::to_string(t) + ".");
    }
    v.f = (double)v.i;
}
}  // namespace

Gguf::Gguf(const std::string& path) : path_(path)
{
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) WL_THROW(WL_EIO, "Cannot open " + path + ".");
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); WL_THROW(WL_EIO, "Cannot stat " + path + "."); }
    len_ = (size_t)st.st_size;
    if (len_ < 24) { close(fd); WL_THROW(WL_EFORMAT, path + " is not a GGUF file."); }
    void* m = mmap(nullptr, len_, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) WL_THROW(WL_EIO, "Cannot map " + path + ".");
    map_ = (uint8_t*)m;
    try {
        Reader r{map_, map_ + len_, path_};
        if (r.get<uint32_t>() != 0x46554747u) WL_THROW(WL_EFORMAT, path + " is not a GGUF file.");
        const uint32_t version = r.get<uint32_t>();
        if (version < 2 || version > 3) WL_THROW(WL_EFORMAT, path + ": unsupported GGUF version " + std::to_string(version) + ".");
        const int64_t nt = r.get<int64_t>(), nkv = r.get<int64_t>();
        if (nt < 0 || nkv < 0 || nt > 1000000 || nkv > 1000000) WL_THROW(WL_EFORMAT, path + ": bad tensor or key count.");
        int64_t alignment = 32;
        for (int64_t i = 0; i < nkv; ++i) {
            const std::string key = r.str();
            GgufValue v;
            v.type = (int)r.get<int32_t>();
            if (v.type == 9) {
                const int at = (int)r.get<int32_t>();
                const int64_t n = r.get<int64_t>();
                if (n < 0 || n > INT32_MAX) WL_THROW(WL_EFORMAT, path + ": bad GGUF array length.");
                if (at == 8) for (int64_t j = 0; j < n; ++j) r.str();
                else {
                    const int sz = scalar_size(at);
                    if (sz < 0) WL_THROW(WL_EFORMAT, path + ": unsupported GGUF array type.");
                    r.need((size_t)(sz * n));
                    r.p += sz * n;
                }
                v.i = n;
            } else read_scalar(r, v.type, v);
            if (key == "general.alignment") alignment = v.i;
            if (!kv_.count(key)) kv_[key] = v;
        }
        if (alignment <= 0 || (alignment & (alignment - 1)) != 0) WL_THROW(WL_EFORMAT, path + ": general.alignment must be a power of two.");
        for (int64_t i = 0; i < nt; ++i) {
            GgufTensor t;
            t.name = r.str();
            const uint32_t nd = r.get<uint32_t>();
            if (nd == 0 || nd > 4) WL_THROW(WL_EFORMAT, "Tensor " + t.name + " has " + std::to_string(nd) + " dims.");
            t.ndims = (int)nd;
            for (uint32_t d = 0; d < nd; ++d) {
                t.dims[d] = r.get<int64_t>();
                if (t.dims[d] <= 0) WL_THROW(WL_EFORMAT, "Tensor " + t.name + " has a non-positive dim.");
            }
            t.type = (int)r.get<int32_t>();
            t.offset = (int64_t)r.get<uint64_t>();
            if (by_name_.count(t.name)) WL_THROW(WL_EFORMAT, "Duplicate tensor " + t.name + ".");
            by_name_[t.name] = tensors_.size();
            tensors_.push_back(t);
        }
        const int64_t data_off = ((int64_t)(r.p - map_) + alignment - 1) / alignment * alignment;
        for (GgufTensor& t : tensors_) {
            int bs = 0, ts = 0;
            if (!layout(t.type, &bs, &ts))
                WL_THROW(WL_EUNSUPPORTED, "Tensor " + t.name + " uses type " + std::to_string(t.type) + ", which Windlass cannot read yet.");
            if (t.dims[0] % bs != 0) WL_THROW(WL_EFORMAT, "Tensor " + t.name + " row is not a multiple of the block size.");
            t.size = t.elements() / bs * ts;
            t.offset += data_off;
            if (t.offset + t.size > (int64_t)len_) WL_THROW(WL_EFORMAT, "Tensor " + t.name + " extends past the end of " + path + ".");
        }
    } catch (...) {
        munmap(map_, len_);
        map_ = nullptr;
        throw;
    }
}

Gguf::~Gguf()
{
    if (map_) munmap(map_, len_);
}

const GgufTensor* Gguf::find(const std::string& name) const
{
    auto it = by_name_.find(name);
    return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

int64_t Gguf::get_int(const std::string& key, int64_t dflt) const
{
    auto it = kv_.find(key);
    return it == kv_.end() || it->second.type == 8 || it->second.type == 9 ? dflt : it->second.i;
}

float Gguf::get_float(const std::string& key, float dflt) const
{
    auto it = kv_.find(key);
    return it == kv_.end() || it->second.type == 8 || it->second.type == 9 ? dflt : (float)it->second.f;
}

std::string Gguf::get_string(const std::string& key, const std::string& dflt) const
{
    auto it = kv_.find(key);
    return it == kv_.end() || it->second.type != 8 ? dflt : it->second.s;
}

bool Gguf::get_bool(const std::string& key, bool dflt) const
{
    auto it = kv_.find(key);
    return it == kv_.end() || it->second.type == 8 || it->second.type == 9 ? dflt : it->second.i != 0;
}

}  // namespace wl
