// Strata pack reader (host code): parses ds4.txt and tensors.txt, opens the GGUF shards
// and reads tensor bytes with pread. The checks are those of crosslane's PackSource
// (engine/strata/sycl/stage/wiring/pack_source.cpp:144-185): model_dir present, format
// "gguf", well-formed and unique tensor lines, no shard index gap, every extent inside its
// shard.
#include <cerrno>
#include <fcntl.h>
#include <fstream>
#include <map>
#include <sstream>
#include <sys/stat.h>
#include <unistd.h>

#include "clb_host.h"
#include "clb_pack_io.h"

struct clb_strata_pack {
    std::string dir, model_dir;
    std::map<std::string, std::string> kv;
    std::vector<std::string> files;
    std::vector<int> fds;
    std::vector<uint64_t> sizes;
    std::map<std::string, clb::PackTensor> tensors;
    ~clb_strata_pack() {
        for (int fd : fds)
            if (fd >= 0) ::close(fd);
    }
};

namespace {
std::string slurp(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    require(bool(f), CLB_E_INVALID, "cannot read %s", path.c_str());
    std::ostringstream s;
    s << f.rdbuf();
    return s.str();
}
}  // namespace

namespace clb {

const PackTensor* pack_find(const clb_strata_pack* p, const std::string& name) {
    auto it = p->tensors.find(name);
    return it == p->tensors.end() ? nullptr : &it->second;
}

std::string pack_meta(const clb_strata_pack* p, const std::string& key) {
    auto it = p->kv.find(key);
    return it == p->kv.end() ? std::string() : it->second;
}

void pack_read(const clb_strata_pack* p, const PackTensor& t, uint64_t offset, void* dst, uint64_t bytes) {
    require(offset <= t.bytes && bytes <= t.bytes - offset, CLB_E_INVALID, "read past the tensor's extent");
    uint8_t* d = static_cast<uint8_t*>(dst);
    uint64_t done = 0;
    while (done < bytes) {
        const ssize_t r = ::pread(p->fds[(size_t)t.file], d + done, (size_t)(bytes - done), (off_t)(t.offset + offset + done));
        if (r < 0 && errno == EINTR) continue;
        require(r > 0, CLB_E_INVALID, "shard read failed (%s)", r < 0 ? std::strerror(errno) : "end of file");
        done += (uint64_t)r;
    }
}

int pack_expert_type(const std::string& dtype) {
    return dtype == "IQ2_XXS" ? 16 : dtype == "IQ2_XS" ? 17 : dtype == "IQ1_M" ? 29 : 0;
}

}  // namespace clb

extern "C" {

int32_t clb_strata_pack_open(const char* dir, clb_strata_pack** out, clb_error_v1* err) {
    if (!dir || !out) return fail(err, CLB_E_INVALID, "null pack directory/output");
    *out = nullptr;
    auto* p = new (std::nothrow) clb_strata_pack();
    if (!p) return fail(err, CLB_E_NOMEM, "host allocation failed");
    const int32_t rc = guarded(err, [&] {
        p->dir = dir;
        const std::string ds4 = slurp(p->dir + "/ds4.txt"), tensors = slurp(p->dir + "/tensors.txt");
        {
            std::istringstream f(ds4);
            std::string line;
            while (std::getline(f, line)) {
                const size_t sp = line.find(' ');
                if (sp != std::string::npos) p->kv[line.substr(0, sp)] = line.substr(sp + 1);
            }
        }
        p->model_dir = clb::pack_meta(p, "model_dir");
        require(!p->model_dir.empty(), CLB_E_INVALID, "ds4.txt: model_dir missing");
        require(clb::pack_meta(p, "format") == "gguf", CLB_E_UNSUPPORTED, "only the GGUF pack format is admitted");
        if (p->model_dir[0] != '/') p->model_dir = p->dir + "/" + p->model_dir;  // relative to the pack
        {
            std::istringstream f(tensors);
            std::string line;
            while (std::getline(f, line)) {
                std::istringstream s(line);
                std::string tag;
                s >> tag;
                if (tag == "file") {
                    int i = -1;
                    std::string name;
                    s >> i >> name;
                    require(i >= 0 && i < (1 << 20) && !name.empty(), CLB_E_INVALID, "tensors.txt: bad file line");
                    if ((int)p->files.size() <= i) p->files.resize((size_t)i + 1);
                    p->files[(size_t)i] = name;
                    continue;
                }
                if (tag != "t") continue;
                std::string name;
                clb::PackTensor x;
                s >> name >> x.dtype >> x.file >> x.offset >> x.bytes;
                require(!s.fail() && !name.empty(), CLB_E_INVALID, "tensors.txt: bad tensor line");
                int64_t d;
                while (s >> d) x.shape.push_back(d);
                require(p->tensors.emplace(name, x).second, CLB_E_INVALID, "tensors.txt: duplicate tensor %s",
                        name.c_str());
            }
        }
        for (const auto& fn : p->files) {
            require(!fn.empty(), CLB_E_INVALID, "tensors.txt: file index gap");
            const std::string path = p->model_dir + "/" + fn;
            const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
            require(fd >= 0, CLB_E_INVALID, "cannot open shard %s", path.c_str());
            p->fds.push_back(fd);
            struct stat st{};
            require(::fstat(fd, &st) == 0, CLB_E_INVALID, "stat shard %s", path.c_str());
            p->sizes.push_back((uint64_t)st.st_size);
        }
        for (const auto& kv : p->tensors) {
            const auto& t = kv.second;
            require(t.file >= 0 && (size_t)t.file < p->fds.size(), CLB_E_INVALID, "tensor %s names an unknown shard",
                    kv.first.c_str());
            const uint64_t size = p->sizes[(size_t)t.file];
            require(t.offset <= size && t.bytes <= size - t.offset, CLB_E_INVALID, "tensor %s extent past shard end",
                    kv.first.c_str());
        }
    });
    if (rc != CLB_OK) {
        delete p;
        return rc;
    }
    *out = p;
    return CLB_OK;
}

void clb_strata_pack_close(clb_strata_pack* pack) { delete pack; }

int32_t clb_strata_pack_meta(const clb_strata_pack* pack, const char* key, char* value, size_t cap) {
    if (!pack || !key || !value || cap == 0) return CLB_E_INVALID;
    const std::string v = clb::pack_meta(pack, key);
    if (v.empty() || v.size() + 1 > cap) return CLB_E_INVALID;
    std::memcpy(value, v.c_str(), v.size() + 1);
    return CLB_OK;
}

int32_t clb_strata_pack_tensor(const clb_strata_pack* pack, const char* name, char* dtype, size_t dtype_cap, uint64_t* bytes,
                        int64_t* shape, int32_t shape_cap, int32_t* ndim) {
    if (!pack || !name) return CLB_E_INVALID;
    const clb::PackTensor* t = clb::pack_find(pack, name);
    if (!t) return CLB_E_INVALID;
    if (dtype) {
        if (dtype_cap < t->dtype.size() + 1) return CLB_E_INVALID;
        std::memcpy(dtype, t->dtype.c_str(), t->dtype.size() + 1);
    }
    if (bytes) *bytes = t->bytes;
    if (ndim) *ndim = (int32_t)t->shape.size();
    if (shape)
        for (int32_t i = 0; i < shape_cap && i < (int32_t)t->shape.size(); ++i) shape[i] = t->shape[(size_t)i];
    return CLB_OK;
}

int32_t clb_strata_pack_read(const clb_strata_pack* pack, const char* name, uint64_t offset, void* dst, uint64_t bytes,
                      clb_error_v1* err) {
    if (!pack || !name || (!dst && bytes)) return fail(err, CLB_E_INVALID, "null pack/name/buffer");
    return guarded(err, [&] {
        const clb::PackTensor* t = clb::pack_find(pack, name);
        require(t != nullptr, CLB_E_INVALID, "missing tensor %s", name);
        clb::pack_read(pack, *t, offset, dst, bytes);
    });
}

}  // extern "C"
