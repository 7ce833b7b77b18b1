// Safetensors snapshot reader for the token-mixer weights: the role of the
// reference's shard index (c/st.h:248-479) and of the mixer part of
// model_init (c/qwen.c:433-485). Host code only; included at the end of
// backend.cu. A snapshot directory holds *.safetensors files (read in name
// order); each is an 8-byte little-endian header length, a JSON header
// {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__":
// {...}} and the data. Offsets, shapes and byte spans are checked before any
// read, as the reference does for untrusted files. Tensors are read with
// pread on demand; nothing stays mapped.
#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <map>
#include <string>

namespace {

struct StTensor {
    int fd = -1;
    int64_t off = 0, nbytes = 0;
    int dtype = -1;               // 0 = BF16, 1 = F16, 2 = F32, 3 = I8/U8
    int ndim = 0;
    int64_t shape[8] = {};
};

struct StSet {
    std::vector<int> fds;
    std::map<std::string, StTensor> t;
};

std::vector<StSet *> g_st;        // handle -> snapshot

int st_dtype(const std::string &s)
{
    if (s == "BF16") return 0;
    if (s == "F16") return 1;
    if (s == "F32") return 2;
    if (s == "I8" || s == "U8") return 3;
    return -1;
}

// Minimal JSON reader for the safetensors header (objects, arrays, strings,
// integers); anything else is a format error.
struct Json {
    const char *p, *e;
    bool ok = true;
    void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p; }
    bool eat(char c) { ws(); if (p < e && *p == c) { ++p; return true; } return false; }
    std::string str()
    {
        std::string s;
        if (!eat('"')) { ok = false; return s; }
        while (p < e && *p != '"') {
            if (*p == '\\' && p + 1 < e) { s += p[1]; p += 2; } else s += *p++;
        }
        if (p >= e) { ok = false; return s; }
        ++p;
        return s;
    }
    int64_t num()
    {
        ws();
        int64_t v = 0;
        bool any = false;
        while (p < e && *p >= '0' && *p <= '9') {
            if (v > (INT64_MAX - 9) / 10) { ok = false; return 0; }
            v = v * 10 + (*p++ - '0');
            any = true;
        }
        if (!any) ok = false;
        return v;
    }
    void skip()                                  // any value (for __metadata__)
    {
        ws();
        if (p >= e) { ok = false; return; }
        if (*p == '"') { str(); return; }
        if (*p == '{' || *p == '[') {
            const char close = *p == '{' ? '}' : ']';
            ++p;
            if (eat(close)) return;
            do {
                if (close == '}') { str(); if (!eat(':')) { ok = false; return; } }
                skip();
            } while (ok && eat(','));
            if (!eat(close)) ok = false;
            return;
        }
        while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
    }
};

bool st_parse_header(const char *hdr, size_t n, int fd, int64_t data_start, int64_t fsz, StSet &S, std::string &why)
{
    Json j{hdr, hdr + n};
    if (!j.eat('{')) { why = "header is not a JSON object"; return false; }
    if (j.eat('}')) return true;
    do {
        const std::string name = j.str();
        if (!j.ok || !j.eat(':')) { why = "bad header key"; return false; }
        if (name == "__metadata__") { j.skip(); if (!j.ok) { why = "bad __metadata__"; return false; } continue; }
        StTensor t;
        t.fd = fd;
        std::string dt;
        int64_t b = -1, en = -1;
        bool have_shape = false;
        if (!j.eat('{')) { why = "tensor entry is not an object: " + name; return false; }
        do {
            const std::string k = j.str();
            if (!j.ok || !j.eat(':')) { why = "bad tensor field in " + name; return false; }
            if (k == "dtype") dt = j.str();
            else if (k == "shape") {
                if (!j.eat('[')) { why = "shape is not an array: " + name; return false; }
                have_shape = true;
                if (!j.eat(']')) {
                    do {
                        if (t.ndim == 8) { why = "too many dimensions: " + name; return false; }
                        t.shape[t.ndim++] = j.num();
                    } while (j.ok && j.eat(','));
                    if (!j.eat(']')) { why = "bad shape: " + name; return false; }
                }
            } else if (k == "data_offsets") {
                if (!j.eat('[')) { why = "data_offsets is not an array: " + name; return false; }
                b = j.num();
                if (!j.eat(',')) { why = "bad data_offsets: " + name; return false; }
                en = j.num();
                if (!j.eat(']')) { why = "bad data_offsets: " + name; return false; }
            } else j.skip();
        } while (j.ok && j.eat(','));
        if (!j.ok || !j.eat('}')) { why = "bad tensor entry: " + name; return false; }
        t.dtype = st_dtype(dt);
        if (t.dtype < 0 || !have_shape || b < 0 || en < b || data_start + en > fsz) {
            why = "tensor '" + name + "' has a bad dtype, shape or data_offsets";
            return false;
        }
        int64_t numel = 1;
        for (int d = 0; d < t.ndim; ++d) {
            if (t.shape[d] < 0 || (t.shape[d] != 0 && numel > INT64_MAX / t.shape[d])) {
                why = "tensor '" + name + "' shape overflows";
                return false;
            }
            numel *= t.shape[d];
        }
        const int esz = t.dtype == 2 ? 4 : t.dtype == 3 ? 1 : 2;
        t.off = data_start + b;
        t.nbytes = en - b;
        if (t.nbytes != numel * esz) { why = "tensor '" + name + "' shape disagrees with its byte span"; return false; }
        S.t[name] = t;
    } while (j.ok && j.eat(','));
    if (!j.ok || !j.eat('}')) { why = "header does not close"; return false; }
    return true;
}

StSet *st_get(int h) { return (h >= 0 && h < (int)g_st.size()) ? g_st[h] : nullptr; }

const StTensor *st_find(int h, const char *name)
{
    StSet *S = st_get(h);
    if (!S || !name) return nullptr;
    auto it = S->t.find(name);
    return it == S->t.end() ? nullptr : &it->second;
}

bool st_pread(int fd, void *buf, int64_t n, int64_t off)
{
    char *b = static_cast<char *>(buf);
    while (n > 0) {
        const ssize_t r = pread(fd, b, (size_t)n, (off_t)off);
        if (r <= 0) return false;
        b += r; n -= r; off += r;
    }
    return true;
}

float half_to_f32(uint16_t h)
{
    const uint32_t s = (uint32_t)(h & 0x8000) << 16, ex = (h >> 10) & 0x1f, m = h & 0x3ff;
    uint32_t u;
    if (ex == 0) {
        if (m == 0) u = s;
        else {   // subnormal: normalise
            int e = -1;
            uint32_t mm = m;
            do { ++e; mm <<= 1; } while (!(mm & 0x400));
            u = s | ((uint32_t)(127 - 15 - e) << 23) | ((mm & 0x3ff) << 13);
        }
    } else if (ex == 31) u = s | 0x7f800000u | (m << 13);
    else u = s | ((ex + 127 - 15) << 23) | (m << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

}  // namespace

extern "C" {

int coli_cuda_st_open(const char *snap_dir)
{
    if (!snap_dir) { fail("no snapshot directory"); return -1; }
    DIR *d = opendir(snap_dir);
    if (!d) { fail("cannot open %s", snap_dir); return -1; }
    std::vector<std::string> files;
    while (struct dirent *de = readdir(d)) {
        const std::string n = de->d_name;
        if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.push_back(n);
    }
    closedir(d);
    std::sort(files.begin(), files.end());
    if (files.empty()) { fail("no *.safetensors in %s", snap_dir); return -1; }
    StSet *S = new StSet();
    for (const auto &f : files) {
        const std::string path = std::string(snap_dir) + "/" + f;
        const int fd = open(path.c_str(), O_RDONLY);
        struct stat sst;
        uint64_t hlen = 0;
        std::string why;
        bool good = fd >= 0 && fstat(fd, &sst) == 0;
        const int64_t fsz = good ? (int64_t)sst.st_size : 0;
        if (good) good = fsz >= 8 && st_pread(fd, &hlen, 8, 0) && hlen <= (uint64_t)(fsz - 8) && hlen <= (512ull << 20);
        if (good) {
            std::vector<char> hdr(hlen);
            good = st_pread(fd, hdr.data(), (int64_t)hlen, 8) &&
                   st_parse_header(hdr.data(), hdr.size(), fd, 8 + (int64_t)hlen, fsz, *S, why);
        } else why = "unreadable file or bad header length";
        if (fd >= 0) S->fds.push_back(fd);
        if (!good) {
            for (int x : S->fds) close(x);
            delete S;
            fail("%s: %s", path.c_str(), why.c_str());
            return -1;
        }
    }
    g_st.push_back(S);
    return (int)g_st.size() - 1;
}

void coli_cuda_st_close(int h)
{
    StSet *S = st_get(h);
    if (!S) return;
    for (int x : S->fds) close(x);
    delete S;
    g_st[h] = nullptr;
}

int coli_cuda_st_info(int h, const char *name, long long *shape, int *ndim, int *dtype)
{
    const StTensor *t = st_find(h, name);
    if (!t) return 0;
    if (ndim) *ndim = t->ndim;
    if (dtype) *dtype = t->dtype;
    if (shape) for (int d = 0; d < t->ndim; ++d) shape[d] = t->shape[d];
    return 1;
}

long long coli_cuda_st_read_f32(int h, const char *name, float *out, long long cap)
{
    const StTensor *t = st_find(h, name);
    if (!t) { fail("tensor %s not in the snapshot", name ? name : "(null)"); return -1; }
    if (t->dtype > 2) { fail("tensor %s is not a float tensor", name); return -1; }
    const int64_t n = t->nbytes / (t->dtype == 2 ? 4 : 2);
    if (n > cap) { fail("tensor %s has %lld elements, buffer %lld", name, (long long)n, cap); return -1; }
    std::vector<uint8_t> raw((size_t)t->nbytes);
    if (!st_pread(t->fd, raw.data(), t->nbytes, t->off)) { fail("read of %s failed", name); return -1; }
    for (int64_t i = 0; i < n; ++i) {
        if (t->dtype == 2) memcpy(out + i, raw.data() + 4 * i, 4);
        else {
            uint16_t v;
            memcpy(&v, raw.data() + 2 * i, 2);
            if (t->dtype == 0) { const uint32_t u = (uint32_t)v << 16; memcpy(out + i, &u, 4); }
            else out[i] = half_to_f32(v);
        }
    }
    return n;
}

int coli_cuda_st_dense(int h, const char *name, ColiCudaTensor **tensor)
{
    READY();
    const StTensor *t = st_find(h, name);
    if (!t) return fail("tensor %s not in the snapshot", name ? name : "(null)");
    if (t->ndim != 2 || t->dtype > 2) return fail("tensor %s is not a 2-D float tensor", name);
    const int O = (int)t->shape[0], I = (int)t->shape[1];
    std::vector<float> w((size_t)O * I);
    if (coli_cuda_st_read_f32(h, name, w.data(), (long long)w.size()) < 0) return 0;
    // BF16 sources come back exactly after the round trip through fp32
    return coli_cuda_tensor_ensure(tensor, w.data(), nullptr, 0, I, O, 0);
}

}  // extern "C"
