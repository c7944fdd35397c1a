// st.cu -- host C++: one MoE layer's routed experts from the checkpoint's safetensors
// shards into a host buffer laid out as the device expert bank (no device code).
//
// The checkpoint format (src/io/k3_st.h:7-13 of the reference): [8-byte little-endian N]
// [N bytes of JSON header][data]; each header entry is {"dtype", "shape", "data_offsets":
// [start, end]} with offsets relative to the end of the header; "__metadata__" may appear.
// A routed expert is six U8 tensors (src/io/k3_load.h:1-22, names src/io/k3_load.c:11):
//   language_model.model.layers.<layer>.block_sparse_moe.experts.<e>.<w>.weight_packed
//   language_model.model.layers.<layer>.block_sparse_moe.experts.<e>.<w>.weight_scale
// for w = w1, w2, w3, with w1/w3 [I][L/2] + [I][L/32] and w2 [L][I/2] + [L][I/32]. The
// device bank keeps them in the same order (k3gpu_bank_layout), so each expert lands with
// one read per tensor, or one read per expert when the six are contiguous in the file.
#include <dirent.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <unordered_map>
#include <vector>

#include "k3gpu.h"

namespace {

struct Entry {
    int file;
    int64_t off, bytes;      // absolute file offset and length
    std::string dtype;
    std::vector<int64_t> shape;
};

// a JSON scanner for safetensors headers: objects, arrays, strings (with escapes),
// numbers, true/false/null; entries are recorded for objects that have data_offsets
struct Scan {
    const char *p, *e;
    bool ok = true;

    void ws()
    {
        while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) p++;
    }
    bool eat(char c)
    {
        ws();
        if (p < e && *p == c) {
            p++;
            return true;
        }
        return false;
    }
    static int hexv(char c)
    {
        if (c >= '0' && c <= '9') return c - '0';
        if (c >= 'a' && c <= 'f') return c - 'a' + 10;
        if (c >= 'A' && c <= 'F') return c - 'A' + 10;
        return -1;
    }
    void utf8(std::string &s, unsigned cp)
    {
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
    unsigned hex4()
    {
        if (e - p < 4) { ok = false; return 0; }
        unsigned v = 0;
        for (int i = 0; i < 4; i++) {
            const int h = hexv(p[i]);
            if (h < 0) { ok = false; return 0; }
            v = v * 16 + (unsigned)h;
        }
        p += 4;
        return v;
    }
    std::string str()
    {
        std::string s;
        if (!eat('"')) { ok = false; return s; }
        while (p < e && *p != '"') {
            if (*p != '\\') { s += *p++; continue; }
            if (++p >= e) { ok = false; return s; }
            const char c = *p++;
            switch (c) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    unsigned cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && e - p >= 6 && p[0] == '\\' && p[1] == 'u') {
                        p += 2;
                        const unsigned lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(s, cp);
                    break;
                }
                default: ok = false; return s;
            }
        }
        if (p >= e) { ok = false; return s; }
        p++;   // closing quote
        return s;
    }
    bool number(int64_t *v)
    {
        ws();
        const char *q = p;
        if (q < e && (*q == '-' || *q == '+')) q++;
        bool digits = false, integral = true;
        while (q < e && ((*q >= '0' && *q <= '9') || *q == '.' || *q == 'e' || *q == 'E' || *q == '-' || *q == '+')) {
            if (*q >= '0' && *q <= '9') digits = true;
            else integral = false;
            q++;
        }
        if (!digits) { ok = false; return false; }
        if (v) *v = integral ? strtoll(std::string(p, q).c_str(), nullptr, 10) : -1;
        p = q;
        return integral;
    }
    // values nested deeper than this are refused (a malformed header, not a stack overflow)
    static constexpr int MAX_DEPTH = 64;
    void skip_value(int depth = 0)
    {
        ws();
        if (p >= e || depth > MAX_DEPTH) { ok = false; return; }
        if (*p == '"') { str(); return; }
        if (*p == '{') {
            p++;
            if (eat('}')) return;
            do {
                str();
                if (!eat(':')) { ok = false; return; }
                skip_value(depth + 1);
            } while (ok && eat(','));
            if (!eat('}')) ok = false;
            return;
        }
        if (*p == '[') {
            p++;
            if (eat(']')) return;
            do skip_value(depth + 1);
            while (ok && eat(','));
            if (!eat(']')) ok = false;
            return;
        }
        for (const char *lit : {"true", "false", "null"}) {
            const size_t n = strlen(lit);
            if ((size_t)(e - p) >= n && !strncmp(p, lit, n)) { p += n; return; }
        }
        number(nullptr);
    }
    std::vector<int64_t> int_array()
    {
        std::vector<int64_t> v;
        if (!eat('[')) { ok = false; return v; }
        if (eat(']')) return v;
        do {
            int64_t x;
            if (!number(&x)) { ok = false; return v; }
            v.push_back(x);
        } while (ok && eat(','));
        if (!eat(']')) ok = false;
        return v;
    }
    // one tensor entry's object; returns false for objects without data_offsets
    bool entry(Entry *t)
    {
        bool has_off = false;
        if (!eat('{')) { ok = false; return false; }
        if (eat('}')) return false;
        do {
            const std::string k = str();
            if (!eat(':')) { ok = false; return false; }
            if (k == "dtype") t->dtype = str();
            else if (k == "shape") t->shape = int_array();
            else if (k == "data_offsets") {
                const std::vector<int64_t> o = int_array();
                if (o.size() != 2 || o[0] < 0 || o[1] < o[0]) { ok = false; return false; }
                t->off = o[0];
                t->bytes = o[1] - o[0];
                has_off = true;
            } else skip_value();
        } while (ok && eat(','));
        if (!eat('}')) ok = false;
        return ok && has_off;
    }
};

int read_header(int fd, int file, std::unordered_map<std::string, Entry> *index, int64_t *file_bytes)
{
    uint8_t nb[8];
    if (pread(fd, nb, 8, 0) != 8) return K3GPU_EINVAL;
    uint64_t n = 0;
    for (int i = 7; i >= 0; i--) n = (n << 8) | nb[i];
    if (n == 0 || n > (1ull << 30)) return K3GPU_EINVAL;
    std::vector<char> h(n);
    if (pread(fd, h.data(), n, 8) != (ssize_t)n) return K3GPU_EINVAL;
    const off_t end = lseek(fd, 0, SEEK_END);
    *file_bytes = (int64_t)end;
    Scan s{h.data(), h.data() + n};
    if (!s.eat('{')) return K3GPU_EINVAL;
    if (s.eat('}')) return K3GPU_OK;
    do {
        const std::string name = s.str();
        if (!s.ok || !s.eat(':')) return K3GPU_EINVAL;
        Entry t;
        t.file = file;
        t.off = t.bytes = 0;
        if (s.entry(&t)) {
            // data past the file (each term bounded first, so the sum cannot overflow)
            if (t.off > *file_bytes || t.bytes > *file_bytes) return K3GPU_EINVAL;
            t.off += 8 + (int64_t)n;
            if (t.off + t.bytes > *file_bytes) return K3GPU_EINVAL;
            (*index)[name] = t;
        }
    } while (s.ok && s.eat(','));
    return (s.ok && s.eat('}')) ? K3GPU_OK : K3GPU_EINVAL;
}

}  // namespace

extern "C" int k3_bank_read_safetensors(const char *const *files, int n_files, int layer, int e0, int n, int L, int I,
                                        uint8_t *host_bank, size_t host_bytes)
{
    if (!files || n_files <= 0 || layer < 0 || e0 < 0 || n <= 0 || e0 > (1 << 20) || n > (1 << 20) || !host_bank)
        return K3GPU_EINVAL;
    if (L <= 0 || I <= 0 || L % 32 || I % 32) return K3GPU_EINVAL;
    K3GpuExpertBank lay;
    memset(&lay, 0, sizeof lay);
    k3gpu_bank_layout(&lay, L, I);
    if ((uint64_t)n * (uint64_t)lay.stride > host_bytes) return K3GPU_ECAPACITY;
    int st = K3GPU_OK;
    std::vector<int> fds;
    std::unordered_map<std::string, Entry> index;
    for (int f = 0; f < n_files && st == K3GPU_OK; f++) {
        const int fd = files[f] ? open(files[f], O_RDONLY) : -1;
        if (fd < 0) { st = K3GPU_EINVAL; break; }
        fds.push_back(fd);
        int64_t fb = 0;
        st = read_header(fd, f, &index, &fb);
    }
    // the six tensors of an expert in run order, with their shapes and bank offsets
    struct Part {
        const char *w, *kind;
        int64_t rows, cols, dst;
    };
    const Part parts[6] = {{"w1", "weight_packed", I, L / 2, lay.p1}, {"w1", "weight_scale", I, L / 32, lay.s1},
                           {"w2", "weight_packed", L, I / 2, lay.p2}, {"w2", "weight_scale", L, I / 32, lay.s2},
                           {"w3", "weight_packed", I, L / 2, lay.p3}, {"w3", "weight_scale", I, L / 32, lay.s3}};
    char name[256];
    for (int e = e0; e < e0 + n && st == K3GPU_OK; e++) {
        uint8_t *run = host_bank + (size_t)(e - e0) * (size_t)lay.stride;
        for (const Part &pt : parts) {
            snprintf(name, sizeof name, "language_model.model.layers.%d.block_sparse_moe.experts.%d.%s.%s", layer, e,
                     pt.w, pt.kind);
            const auto it = index.find(name);
            if (it == index.end()) { st = K3GPU_EINVAL; break; }
            const Entry &t = it->second;
            if (t.dtype != "U8" || t.shape.size() != 2 || t.shape[0] != pt.rows || t.shape[1] != pt.cols ||
                t.bytes != pt.rows * pt.cols) {
                st = K3GPU_EINVAL;
                break;
            }
            if (pread(fds[t.file], run + pt.dst, (size_t)t.bytes, t.off) != (ssize_t)t.bytes) {
                st = K3GPU_EINVAL;
                break;
            }
        }
    }
    for (int fd : fds) close(fd);
    return st;
}

// ---- a tensor index over a shard set (the reference's k3_st_open / find / read) --------
// One open over the shards' headers, then any tensor by name: the trunk's bf16 and fp32
// tensors as well as the experts' U8 runs, read raw with pread (no mapping, so resident
// memory stays what the caller holds).
struct K3StIndex {
    std::vector<int> fds;
    std::unordered_map<std::string, Entry> index;
    std::vector<std::string> names;   // discovery order: shard by shard, header order
};

namespace {

int dtype_code(const std::string &d)
{
    if (d == "U8") return K3_ST_U8;
    if (d == "BF16") return K3_ST_BF16;
    if (d == "F16") return K3_ST_F16;
    if (d == "F32") return K3_ST_F32;
    return K3_ST_UNKNOWN;
}

// header keys in file order, for the discovery order of the index
std::vector<std::string> header_names(int fd)
{
    std::vector<std::string> out;
    uint8_t nb[8];
    if (pread(fd, nb, 8, 0) != 8) return out;
    uint64_t n = 0;
    for (int i = 7; i >= 0; i--) n = (n << 8) | nb[i];
    if (n == 0 || n > (1ull << 30)) return out;
    std::vector<char> h(n);
    if (pread(fd, h.data(), n, 8) != (ssize_t)n) return out;
    Scan s{h.data(), h.data() + n};
    if (!s.eat('{') || s.eat('}')) return out;
    do {
        std::string name = s.str();
        if (!s.ok || !s.eat(':')) break;
        s.skip_value();
        if (name != "__metadata__") out.push_back(name);
    } while (s.ok && s.eat(','));
    return out;
}

}  // namespace

extern "C" K3StIndex *k3_st_open_files(const char *const *files, int n_files)
{
    if (!files || n_files <= 0) return nullptr;
    K3StIndex *s = new K3StIndex;
    bool ok = true;
    for (int f = 0; f < n_files && ok; f++) {
        const int fd = files[f] ? open(files[f], O_RDONLY) : -1;
        if (fd < 0) { ok = false; break; }
        s->fds.push_back(fd);
        std::unordered_map<std::string, Entry> one;
        int64_t fb = 0;
        if (read_header(fd, f, &one, &fb) != K3GPU_OK) { ok = false; break; }
        for (const std::string &name : header_names(fd)) {
            const auto it = one.find(name);
            if (it == one.end()) continue;                   // an entry without data_offsets
            // a name already seen, in another shard or earlier in this one: the set is broken
            if (!s->index.emplace(name, it->second).second) { ok = false; break; }
            s->names.push_back(name);
        }
    }
    if (!ok) {
        k3_st_close(s);
        return nullptr;
    }
    return s;
}

extern "C" K3StIndex *k3_st_open(const char *dir)
{
    if (!dir) return nullptr;
    DIR *d = opendir(dir);
    if (!d) return nullptr;
    std::vector<std::string> paths;
    while (const dirent *e = readdir(d)) {
        const std::string n = e->d_name;
        const std::string ext = ".safetensors";
        if (n.size() > ext.size() && n.compare(n.size() - ext.size(), ext.size(), ext) == 0)
            paths.push_back(std::string(dir) + "/" + n);
    }
    closedir(d);
    if (paths.empty()) return nullptr;
    std::sort(paths.begin(), paths.end());                   // shard order by name
    std::vector<const char *> ptrs;
    for (const std::string &p : paths) ptrs.push_back(p.c_str());
    return k3_st_open_files(ptrs.data(), (int)ptrs.size());
}

extern "C" void k3_st_close(K3StIndex *s)
{
    if (!s) return;
    for (int fd : s->fds) close(fd);
    delete s;
}

extern "C" int k3_st_count(const K3StIndex *s) { return s ? (int)s->names.size() : 0; }

extern "C" const char *k3_st_name(const K3StIndex *s, int i)
{
    if (!s || i < 0 || i >= (int)s->names.size()) return nullptr;
    return s->names[(size_t)i].c_str();
}

extern "C" int k3_st_find(const K3StIndex *s, const char *name, K3StTensorInfo *info)
{
    if (!s || !name || !info) return K3GPU_EINVAL;
    const auto it = s->index.find(name);
    if (it == s->index.end()) return K3GPU_EINVAL;
    const Entry &t = it->second;
    if (t.shape.size() > 8) return K3GPU_EINVAL;
    memset(info, 0, sizeof *info);
    info->dtype = dtype_code(t.dtype);
    snprintf(info->dtype_name, sizeof info->dtype_name, "%s", t.dtype.c_str());
    info->ndim = (int)t.shape.size();
    for (size_t i = 0; i < t.shape.size(); i++) info->shape[i] = t.shape[i];
    info->shard = t.file;
    info->nbytes = t.bytes;
    return K3GPU_OK;
}

extern "C" int64_t k3_st_read(const K3StIndex *s, const char *name, void *buf, size_t buf_bytes)
{
    if (!s || !name || !buf) return K3GPU_EINVAL;
    const auto it = s->index.find(name);
    if (it == s->index.end()) return K3GPU_EINVAL;
    const Entry &t = it->second;
    if ((uint64_t)t.bytes > buf_bytes) return K3GPU_ECAPACITY;
    int64_t done = 0;
    while (done < t.bytes) {
        const ssize_t r = pread(s->fds[(size_t)t.file], (char *)buf + done, (size_t)(t.bytes - done), t.off + done);
        if (r <= 0) return K3GPU_EINVAL;
        done += r;
    }
    return t.bytes;
}
