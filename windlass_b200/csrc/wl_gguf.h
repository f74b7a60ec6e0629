// GGUF v2/v3 reader (GgufModelFile, src/Gguf.cs:104-270): metadata and the tensor index of one file, with the
// tensor bytes reachable through a read-only mapping of the file.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace wl {

struct GgufValue {
    int type = -1;          // GgufType (src/Gguf.cs:12-16)
    int64_t i = 0;
    double f = 0;
    std::string s;
};

struct GgufTensor {
    std::string name;
    int64_t dims[4] = {1, 1, 1, 1};
    int ndims = 0;
    int type = -1;
    int64_t offset = 0;     // absolute offset in the file
    int64_t size = 0;       // bytes
    int64_t elements() const { return dims[0] * dims[1] * dims[2] * dims[3]; }
    int cols() const { return (int)dims[0]; }
    int rows() const { return (int)(elements() / dims[0]); }
    int experts() const { return (int)(dims[2] * dims[3]); }
};

class Gguf {
public:
    // Throws wl::Error (WL_EIO, WL_EFORMAT, WL_EUNSUPPORTED) like GgufModelFile.ReadHeader.
    explicit Gguf(const std::string& path);
    ~Gguf();
    Gguf(const Gguf&) = delete;
    Gguf& operator=(const Gguf&) = delete;

    const GgufTensor* find(const std::string& name) const;
    bool has(const std::string& key) const { return kv_.count(key) != 0; }
    int64_t get_int(const std::string& key, int64_t dflt) const;
    float get_float(const std::string& key, float dflt) const;
    std::string get_string(const std::string& key, const std::string& dflt) const;
    bool get_bool(const std::string& key, bool dflt) const;
    const uint8_t* data(const GgufTensor& t) const { return map_ + t.offset; }
    const std::vector<GgufTensor>& tensors() const { return tensors_; }
    const std::string& path() const { return path_; }

private:
    std::string path_;
    uint8_t* map_ = nullptr;
    size_t len_ = 0;
    std::map<std::string, GgufValue> kv_;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, size_t> by_name_;
};

}  // namespace wl
