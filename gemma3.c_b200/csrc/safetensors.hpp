// safetensors.hpp - read-only index of a SafeTensors checkpoint directory
// (host code).  Replaces the reference's st_load / st_find_tensor /
// st_get_tensor_data (gemma3_safetensors.c:393-516) for the device upload
// path: every *.safetensors file of the directory (sorted by name, as the
// reference does) is memory-mapped, its header parsed, and tensors are found
// by name.
//
// File format: an 8-byte little-endian header length n, then n bytes of JSON
// {"name": {"dtype": "BF16", "shape": [d0, ...], "data_offsets": [b, e]},
//  ..., "__metadata__": {...}}, then the data; offsets are relative to the
// first byte after the header.
#pragma once
#include <dirent.h>
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

namespace g3st {

struct Tensor {
    std::string dtype;
    std::vector<int64_t> shape;
    const unsigned char *data = nullptr;
    size_t bytes = 0;
};

// Minimal JSON reader for the header: objects, arrays, strings (with the
// usual escapes), integers; anything else inside __metadata__ is skipped.
class Json {
  public:
    Json(const char *s, size_t n) : p_(s), e_(s + n) {}
    bool ok() const { return ok_; }
    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }
    bool eat(char c) {
        ws();
        if (p_ < e_ && *p_ == c) {
            ++p_;
            return true;
        }
        return false;
    }
    bool peek(char c) {
        ws();
        return p_ < e_ && *p_ == c;
    }
    bool str(std::string &out) {
        out.clear();
        if (!eat('"')) return fail();
        while (p_ < e_ && *p_ != '"') {
            if (*p_ == '\\') {
                if (++p_ >= e_) return fail();
                const char c = *p_;
                if (c == 'u') {  // keep \uXXXX verbatim: tensor names are ASCII
                    if (e_ - p_ < 5) return fail();
                    out.append(p_ - 1, 6);
                    p_ += 5;
                    continue;
                }
                out.push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c == 'r' ? '\r' : c == 'b' ? '\b' : c == 'f' ? '\f' : c);
                ++p_;
            } else {
                out.push_back(*p_++);
            }
        }
        if (p_ >= e_) return fail();
        ++p_;
        return true;
    }
    bool integer(int64_t &v) {
        ws();
        bool neg = false;
        if (p_ < e_ && *p_ == '-') {
            neg = true;
            ++p_;
        }
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return fail();
        v = 0;
        while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
            if (v > (INT64_MAX - 9) / 10) return fail();
            v = v * 10 + (*p_++ - '0');
        }
        if (neg) v = -v;
        return true;
    }
    bool skip() {  // any value
        ws();
        if (p_ >= e_) return fail();
        if (*p_ == '"') {
            std::string t;
            return str(t);
        }
        if (*p_ == '{' || *p_ == '[') {
            const char close = *p_ == '{' ? '}' : ']';
            const bool obj = *p_ == '{';
            ++p_;
            if (eat(close)) return true;
            do {
                if (obj) {
                    std::string k;
                    if (!str(k) || !eat(':')) return fail();
                }
                if (!skip()) return false;
            } while (eat(','));
            return eat(close) || fail();
        }
        while (p_ < e_ && *p_ != ',' && *p_ != '}' && *p_ != ']') ++p_;  // number / true / false / null
        return true;
    }
    bool fail() {
        ok_ = false;
        return false;
    }

  private:
    const char *p_, *e_;
    bool ok_ = true;
};

class Index {
  public:
    ~Index() {
        for (auto &m : maps_) munmap(m.first, m.second);
    }
    // Opens every *.safetensors file of `dir`; false with `err` set on failure.
    bool open(const char *dir, std::string &err) {
        DIR *d = opendir(dir);
        if (!d) {
            err = std::string("cannot open directory ") + dir;
            return false;
        }
        std::vector<std::string> files;
        while (dirent *e = readdir(d)) {
            const std::string n = e->d_name;
            const std::string suf = ".safetensors";
            if (n.size() > suf.size() && n.compare(n.size() - suf.size(), suf.size(), suf) == 0)
                files.push_back(std::string(dir) + "/" + n);
        }
        closedir(d);
        if (files.empty()) {
            err = std::string("no .safetensors file in ") + dir;
            return false;
        }
        std::sort(files.begin(), files.end());
        for (const auto &f : files)
            if (!open_file(f, err)) return false;
        return true;
    }
    const Tensor *find(const std::string &name) const {
        auto it = tensors_.find(name);
        return it == tensors_.end() ? nullptr : &it->second;
    }
    size_t size() const { return tensors_.size(); }

  private:
    bool open_file(const std::string &path, std::string &err) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) {
            err = "cannot open " + path;
            return false;
        }
        struct stat st;
        if (fstat(fd, &st) != 0 || st.st_size < 8) {
            ::close(fd);
            err = path + ": too short for a SafeTensors header";
            return false;
        }
        void *m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        ::close(fd);
        if (m == MAP_FAILED) {
            err = "cannot map " + path;
            return false;
        }
        maps_.push_back({m, (size_t)st.st_size});
        const unsigned char *base = (const unsigned char *)m;
        uint64_t hlen = 0;
        for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | base[i];
        if (hlen > (uint64_t)st.st_size - 8) {
            err = path + ": header length beyond the file";
            return false;
        }
        const unsigned char *data = base + 8 + hlen;
        const size_t data_len = (size_t)st.st_size - 8 - hlen;
        Json j((const char *)base + 8, hlen);
        if (!j.eat('{')) {
            err = path + ": header is not a JSON object";
            return false;
        }
        if (!j.eat('}')) {
            do {
                std::string name;
                if (!j.str(name) || !j.eat(':')) break;
                if (name == "__metadata__") {
                    if (!j.skip()) break;
                    continue;
                }
                Tensor t;
                int64_t b0 = -1, b1 = -1;
                if (!j.eat('{')) break;
                do {
                    std::string key;
                    if (!j.str(key) || !j.eat(':')) break;
                    if (key == "dtype") {
                        j.str(t.dtype);
                    } else if (key == "shape") {
                        if (!j.eat('[')) break;
                        if (!j.eat(']')) {
                            do {
                                int64_t v;
                                if (!j.integer(v)) break;
                                t.shape.push_back(v);
                            } while (j.eat(','));
                            if (!j.eat(']')) j.fail();
                        }
                    } else if (key == "data_offsets") {
                        if (!j.eat('[') || !j.integer(b0) || !j.eat(',') || !j.integer(b1) || !j.eat(']')) j.fail();
                    } else {
                        j.skip();
                    }
                } while (j.ok() && j.eat(','));
                if (!j.ok() || !j.eat('}')) {
                    j.fail();
                    break;
                }
                if (b0 < 0 || b1 < b0 || (uint64_t)b1 > data_len) {
                    err = path + ": tensor " + name + " has offsets outside the file";
                    return false;
                }
                t.data = data + b0;
                t.bytes = (size_t)(b1 - b0);
                tensors_[name] = t;
            } while (j.ok() && j.eat(','));
            if (!j.ok() || !j.eat('}')) {
                err = path + ": malformed header JSON";
                return false;
            }
        }
        return true;
    }

    std::vector<std::pair<void *, size_t>> maps_;
    std::map<std::string, Tensor> tensors_;
};

}  // namespace g3st
