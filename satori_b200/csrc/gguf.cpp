// gguf.cpp -- native GGUF v3 catalogue reader and model loader, and the STQ2 (Ternary2 file) reader.
//
// The catalogue rules follow GgufFile.Parse (src/Satori.Formats.Gguf/GgufFile.cs:78-176) and
// GgufCursor (GgufCursor.cs:7-55): little-endian v3 only, key / name / string limits, the supported
// tensor types (F32, F16, Q4_0, Q8_0, Q4_K, Q6_K), alignment, canonical tensor order, and the same
// split of failures into InvalidDataException (SATORI_ERR_INVALID_DATA) and NotSupportedException
// (SATORI_ERR_NOT_SUPPORTED).  The file is mapped read-only; tensor payloads are read straight from the
// mapping when a matrix or a session uploads them (once, unchanged in layout).
//
// The model description follows ModelConfig (src/Satori.Core/Model/ModelConfig.cs: keys resolved
// against the architecture prefix) and DenseTransformerAdapter.Validate
// (src/Satori.Core/Model/DenseTransformerAdapter.cs:12-121): qwen2 / qwen3 dense decoders.
#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "../../include/satori_cuda.h"

namespace satori {
int set_error(int status, const char *fmt, ...);
}
using satori::set_error;

namespace {

constexpr int64_t kHeaderLimit = 256LL * 1024 * 1024;   // GgufCursor.Skip: header limit 256 MiB
constexpr int64_t kFileLimit = 1LL << 40;                // GgufFile: 1 TiB

struct GgufError {
    int status;
    std::string message;
};

[[noreturn]] void bad(int64_t pos, const std::string &what)
{
    throw GgufError{SATORI_ERR_INVALID_DATA, "GGUF at byte " + std::to_string(pos) + ": " + what + "."};
}

[[noreturn]] void unsupported(const std::string &what) { throw GgufError{SATORI_ERR_NOT_SUPPORTED, what}; }

// Strict UTF-8 (no overlong forms, no surrogates, at most U+10FFFF), as .NET's throwing decoder.
bool valid_utf8(const uint8_t *s, int64_t n)
{
    int64_t i = 0;
    while (i < n) {
        const uint8_t c = s[i];
        if (c < 0x80) {
            ++i;
            continue;
        }
        int len;
        uint32_t cp;
        if ((c & 0xE0) == 0xC0) len = 2, cp = c & 0x1F;
        else if ((c & 0xF0) == 0xE0) len = 3, cp = c & 0x0F;
        else if ((c & 0xF8) == 0xF0) len = 4, cp = c & 0x07;
        else return false;
        if (i + len > n) return false;
        for (int k = 1; k < len; ++k) {
            if ((s[i + k] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (s[i + k] & 0x3F);
        }
        if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000)) return false;
        if (cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
        i += len;
    }
    return true;
}

struct Cursor {
    const uint8_t *data;
    int64_t length;
    int64_t pos = 0;

    void skip(int64_t n)
    {
        if (n < 0 || n > length - pos) bad(pos, "Truncated value");
        if (n > kHeaderLimit - pos) unsupported("Header limit: 256 MiB.");
        pos += n;
    }
    uint64_t unsigned_(int size)
    {
        const int64_t start = pos;
        skip(size);
        uint64_t v = 0;
        for (int k = size - 1; k >= 0; --k) v = (v << 8) | data[start + k];
        return v;
    }
    int64_t count(uint64_t v)
    {
        if (v > (uint64_t)INT64_MAX) bad(pos, "Integer exceeds Int64");
        return (int64_t)v;
    }
    std::string string(int64_t limit)
    {
        const int64_t n = count(unsigned_(8));
        if (n > limit) unsupported("String byte limit: " + std::to_string(limit) + " at " + std::to_string(pos) + ".");
        const int64_t start = pos;
        skip(n);
        if (!valid_utf8(data + start, n)) bad(pos, "Invalid UTF-8");
        return std::string(reinterpret_cast<const char *>(data + start), (size_t)n);
    }
};

struct Meta {
    std::string key;
    uint32_t type;
    int64_t offset, length;   // value bytes (for arrays: from the element type on)
    uint32_t elem_type;
    int64_t count;
};

struct TensorRec {
    std::string name;
    int rank;
    int64_t dims[4];
    uint32_t type;
    int64_t offset;           // absolute file offset of the payload
    int64_t bytes;
};

int64_t align_up(int64_t v, int64_t a)
{
    if (v > INT64_MAX - (a - 1)) throw GgufError{SATORI_ERR_INVALID_DATA, "GGUF: offset or dimension overflow."};
    return (v + a - 1) & ~(a - 1);
}

int64_t checked_mul(int64_t a, int64_t b)
{
    int64_t r;
    if (__builtin_mul_overflow(a, b, &r)) throw GgufError{SATORI_ERR_INVALID_DATA, "GGUF: offset or dimension overflow."};
    return r;
}

int64_t checked_add(int64_t a, int64_t b)
{
    int64_t r;
    if (__builtin_add_overflow(a, b, &r)) throw GgufError{SATORI_ERR_INVALID_DATA, "GGUF: offset or dimension overflow."};
    return r;
}

void check_scalar_type(uint32_t t)
{
    if (t > 12 || t == 9) unsupported("Metadata scalar type " + std::to_string(t) + " is unsupported.");
}

void skip_scalar(Cursor &c, uint32_t t)
{
    check_scalar_type(t);
    if (t == 8) {
        (void)c.string(16 * 1024 * 1024);
        return;
    }
    if (t == 7) {
        if (c.unsigned_(1) > 1) bad(c.pos, "Invalid Boolean");
        return;
    }
    c.skip(t <= 1 ? 1 : t <= 3 ? 2 : t <= 6 ? 4 : 8);
}

bool valid_key(const std::string &k)
{
    if (k.empty()) return false;
    size_t start = 0;
    while (true) {
        const size_t dot = k.find('.', start);
        const std::string part = k.substr(start, dot == std::string::npos ? std::string::npos : dot - start);
        if (part.empty()) return false;
        for (char ch : part)
            if (!((ch >= 'a' && ch <= 'z') || (ch >= '0' && ch <= '9') || ch == '_')) return false;
        if (dot == std::string::npos) return true;
        start = dot + 1;
    }
}

// GGUF tensor type -> (block elements, block bytes), GgufFile.cs:137-142.
bool type_geometry(uint32_t t, int *block, int *bytes)
{
    switch (t) {
    case 0: *block = 1, *bytes = 4; return true;      // F32
    case 1: *block = 1, *bytes = 2; return true;      // F16
    case 2: *block = 32, *bytes = 18; return true;    // Q4_0
    case 8: *block = 32, *bytes = 34; return true;    // Q8_0
    case 12: *block = 256, *bytes = 144; return true; // Q4_K
    case 14: *block = 256, *bytes = 210; return true; // Q6_K
    default: return false;
    }
}

}  // namespace

struct satori_gguf {
    int fd = -1;
    const uint8_t *map = nullptr;
    int64_t length = 0;
    std::vector<Meta> meta;
    std::map<std::string, size_t> meta_index;
    std::vector<TensorRec> tensors;
    std::map<std::string, size_t> tensor_index;
    int64_t data_offset = 0;
    std::string architecture;

    ~satori_gguf()
    {
        if (map && map != MAP_FAILED) munmap(const_cast<uint8_t *>(map), (size_t)length);
        if (fd >= 0) close(fd);
    }

    const Meta *find_meta(const std::string &k) const
    {
        auto it = meta_index.find(k);
        return it == meta_index.end() ? nullptr : &meta[it->second];
    }

    // Little-endian scalar of the metadata entry (not arrays, not strings).
    uint64_t raw(const Meta &m) const
    {
        const int size = m.type <= 1 ? 1 : m.type <= 3 ? 2 : m.type <= 7 ? (m.type == 7 ? 1 : 4) : 8;
        uint64_t v = 0;
        for (int k = size - 1; k >= 0; --k) v = (v << 8) | map[m.offset + k];
        return v;
    }
    std::string str(const Meta &m) const
    {
        return std::string(reinterpret_cast<const char *>(map + m.offset + 8), (size_t)(m.length - 8));
    }

    // GgufFile.Get<T>: absent -> fallback; present with another type -> InvalidDataException.
    uint64_t get_uint(const std::string &k, uint32_t type, uint64_t fallback) const
    {
        const Meta *m = find_meta(k);
        if (!m) return fallback;
        if (m->type != type) bad(m->offset, "wrong type for " + k);
        return raw(*m);
    }
    std::string get_string(const std::string &k, const std::string &fallback) const
    {
        const Meta *m = find_meta(k);
        if (!m) return fallback;
        if (m->type != 8) bad(m->offset, "wrong type for " + k);
        return str(*m);
    }

    void parse();
};

void satori_gguf::parse()
{
    Cursor c{map, length};
    if (c.unsigned_(4) != 0x46554747u) bad(c.pos, "Invalid magic");
    if (c.unsigned_(4) != 3) unsupported("Only little-endian GGUF v3 is supported.");
    const int64_t tensor_count = c.count(c.unsigned_(8));
    const int64_t meta_count = c.count(c.unsigned_(8));
    if (tensor_count == 0) unsupported("Tensor count zero is outside the profile.");
    if (tensor_count > 100000 || meta_count > 100000) unsupported("Catalogue count limit: 100000.");
    for (int64_t i = 0; i < meta_count; ++i) {
        const std::string key = c.string(65535);
        if (!valid_key(key)) bad(c.pos, "Invalid metadata key");
        const uint32_t type = (uint32_t)c.unsigned_(4);
        const int64_t start = c.pos;
        uint32_t elem = 0;
        int64_t count = -1;
        if (type == 9) {
            elem = (uint32_t)c.unsigned_(4);
            count = c.count(c.unsigned_(8));
            if (count > 1048576) unsupported("Array count limit: 1048576.");
            check_scalar_type(elem);
            for (int64_t j = 0; j < count; ++j) skip_scalar(c, elem);
        } else {
            skip_scalar(c, type);
        }
        if (meta_index.count(key)) bad(c.pos, "Duplicate metadata key");
        meta_index[key] = meta.size();
        meta.push_back(Meta{key, type, start, c.pos - start, elem, count});
    }
    const uint64_t alignment = get_uint("general.alignment", 4, 32);
    if (alignment == 0 || (alignment & (alignment - 1)) != 0) bad(c.pos, "Invalid alignment");
    if (alignment < 8 || alignment > 4096) unsupported("Alignment range: 8 to 4096.");
    architecture = get_string("general.architecture", "");
    bool arch_ok = !architecture.empty();
    for (char ch : architecture) arch_ok &= (ch >= 'a' && ch <= 'z') || (ch >= '0' && ch <= '9');
    if (!arch_ok) bad(c.pos, "Missing or invalid general.architecture");
    if (get_string("general.type", "model") != "model") unsupported("Only model files are supported.");
    (void)get_uint("general.file_type", 4, 0);
    const uint64_t split_count = get_uint("split.count", 2, 1), split_no = get_uint("split.no", 2, 0);
    if (!(split_count == 0 || split_count == 1) || split_no != 0) unsupported("Sharded GGUF is unsupported.");
    const int32_t split_tensors = (int32_t)(uint32_t)get_uint("split.tensors.count", 5, (uint64_t)(uint32_t)tensor_count);
    if (split_tensors != tensor_count) bad(c.pos, "Invalid split.tensors.count");

    bool quantized = false;
    std::set<std::string> names;
    for (int64_t i = 0; i < tensor_count; ++i) {
        TensorRec t = {};
        t.name = c.string(63);
        if (t.name.empty() || t.name.find('\0') != std::string::npos) bad(c.pos, "Invalid tensor name");
        const uint32_t rank = (uint32_t)c.unsigned_(4);
        if (rank == 0) bad(c.pos, "Zero rank");
        if (rank > 4) unsupported("Tensor rank limit: 4.");
        t.rank = (int)rank;
        int64_t elements = 1;
        for (uint32_t d = 0; d < rank; ++d) {
            t.dims[d] = c.count(c.unsigned_(8));
            if (t.dims[d] == 0) bad(c.pos, "Zero dimension");
            elements = checked_mul(elements, t.dims[d]);
        }
        t.type = (uint32_t)c.unsigned_(4);
        int block, bb;
        if (!type_geometry(t.type, &block, &bb)) unsupported("Tensor type " + std::to_string(t.type) + " is unsupported.");
        quantized |= block != 1;
        if (t.dims[0] % block != 0) bad(c.pos, "Quantized row is not a multiple of " + std::to_string(block));
        t.bytes = checked_mul(elements / block, bb);
        t.offset = c.count(c.unsigned_(8));
        if (t.offset % (int64_t)alignment != 0) bad(c.pos, "Unaligned tensor offset");
        (void)checked_add(t.offset, align_up(t.bytes, (int64_t)alignment));
        if (!names.insert(t.name).second) bad(c.pos, "Duplicate tensor name");
        tensors.push_back(t);
    }
    if (quantized && !find_meta("general.quantization_version")) bad(c.pos, "Missing quantization version");
    if (get_uint("general.quantization_version", 4, 2) != 2) unsupported("Quantization version must be 2.");
    data_offset = align_up(c.pos, (int64_t)alignment);
    c.skip(data_offset - c.pos);
    std::vector<const TensorRec *> by_offset;
    for (const TensorRec &t : tensors) by_offset.push_back(&t);
    std::stable_sort(by_offset.begin(), by_offset.end(),
                     [](const TensorRec *a, const TensorRec *b) { return a->offset < b->offset; });
    int64_t previous_end = 0;
    for (const TensorRec *t : by_offset) {
        const int64_t end = checked_add(t->offset, align_up(t->bytes, (int64_t)alignment));
        if (end > length - data_offset) bad(c.pos, "Tensor data or final padding exceeds file");
        if (t->offset < previous_end) bad(c.pos, "Overlapping tensor ranges");
        previous_end = end;
    }
    int64_t expected = 0;
    for (const TensorRec &t : tensors) {
        if (t.offset != expected) unsupported("Noncanonical tensor gap/order.");
        expected = checked_add(t.offset, align_up(t.bytes, (int64_t)alignment));
    }
    for (size_t i = 0; i < tensors.size(); ++i) {
        tensors[i].offset = checked_add(data_offset, tensors[i].offset);
        tensor_index[tensors[i].name] = i;
    }
}

namespace {

// Maps `path` read-only.  A file longer than `limit` bytes is refused before it is mapped (GgufFile.cs:21).
int map_file(const char *path, int64_t limit, int *fd_out, const uint8_t **map_out, int64_t *len_out)
{
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(SATORI_ERR_ARGUMENT, "cannot open %s: %s", path, strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        return set_error(SATORI_ERR_ARGUMENT, "cannot stat %s", path);
    }
    if ((int64_t)st.st_size > limit) {
        close(fd);
        if (limit == kFileLimit) return set_error(SATORI_ERR_NOT_SUPPORTED, "File limit: 1 TiB.");
        return set_error(SATORI_ERR_NOT_SUPPORTED, "File limit: %lld bytes.", (long long)limit);
    }
    *fd_out = fd;
    *len_out = (int64_t)st.st_size;
    *map_out = nullptr;
    if (st.st_size > 0) {
        void *m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (m == MAP_FAILED) {
            close(fd);
            *fd_out = -1;
            return set_error(SATORI_ERR_ARGUMENT, "cannot map %s", path);
        }
        *map_out = static_cast<const uint8_t *>(m);
    }
    return SATORI_OK;
}

// ModelConfig.TryInt / TryFloat over one metadata entry (ModelConfig.cs:21-60).
bool meta_int(const satori_gguf *g, const std::string &key, int64_t *v)
{
    const Meta *m = g->find_meta(key);
    if (!m || m->type == 9) return false;
    const uint64_t r = m->type == 8 ? 0 : g->raw(*m);
    switch (m->type) {
    case 0: *v = (uint8_t)r; return true;
    case 1: *v = (int8_t)r; return true;
    case 2: *v = (uint16_t)r; return true;
    case 3: *v = (int16_t)r; return true;
    case 4: *v = (uint32_t)r; return true;
    case 5: *v = (int32_t)r; return true;
    case 10: if (r > (uint64_t)INT64_MAX) return false; *v = (int64_t)r; return true;
    case 11: *v = (int64_t)r; return true;
    case 6: {
        float f;
        uint32_t u = (uint32_t)r;
        memcpy(&f, &u, 4);
        if (!(f == std::floor(f)) || f < -9.2e18f || f > 9.2e18f) return false;
        *v = (int64_t)f;
        return true;
    }
    case 12: {
        double d;
        memcpy(&d, &r, 8);
        if (!(d == std::floor(d)) || d < -9.2e18 || d > 9.2e18) return false;
        *v = (int64_t)d;
        return true;
    }
    case 8: {
        const std::string s = g->str(*m);
        char *end = nullptr;
        errno = 0;
        const long long p = strtoll(s.c_str(), &end, 10);
        if (s.empty() || errno || *end) return false;
        *v = p;
        return true;
    }
    default: return false;
    }
}

bool meta_float(const satori_gguf *g, const std::string &key, double *v)
{
    const Meta *m = g->find_meta(key);
    if (!m || m->type == 9 || m->type == 7 || m->type == 8) return false;
    const uint64_t r = g->raw(*m);
    switch (m->type) {
    case 6: {
        float f;
        uint32_t u = (uint32_t)r;
        memcpy(&f, &u, 4);
        *v = f;
        return true;
    }
    case 12: memcpy(v, &r, 8); return true;
    default: {
        int64_t i;
        if (m->type == 10) {
            *v = (double)r;
            return true;
        }
        if (!meta_int(g, key, &i)) return false;
        *v = (double)i;
        return true;
    }
    }
}

bool meta_bool(const satori_gguf *g, const std::string &key, bool *v)
{
    const Meta *m = g->find_meta(key);
    if (!m || m->type != 7) return false;
    *v = g->raw(*m) != 0;
    return true;
}

const TensorRec *tensor(const satori_gguf *g, const std::string &name)
{
    auto it = g->tensor_index.find(name);
    return it == g->tensor_index.end() ? nullptr : &g->tensors[it->second];
}

}  // namespace

extern "C" int satori_gguf_open(const char *path, satori_gguf **out)
{
    if (!path || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    std::unique_ptr<satori_gguf> g(new satori_gguf());
    int rc = map_file(path, kFileLimit, &g->fd, &g->map, &g->length);
    if (rc) return rc;
    if (g->length == 0) return set_error(SATORI_ERR_INVALID_DATA, "GGUF at byte 0: empty file.");
    try {
        g->parse();
    } catch (const GgufError &e) {
        return set_error(e.status, "%s", e.message.c_str());
    }
    *out = g.release();
    return SATORI_OK;
}

extern "C" int satori_gguf_close(satori_gguf *g)
{
    delete g;
    return SATORI_OK;
}

extern "C" int satori_gguf_counts(const satori_gguf *g, int *tensors, int *metadata)
{
    if (!g) return set_error(SATORI_ERR_DISPOSED, "GGUF file is closed");
    if (tensors) *tensors = (int)g->tensors.size();
    if (metadata) *metadata = (int)g->meta.size();
    return SATORI_OK;
}

extern "C" int satori_gguf_tensor_info(const satori_gguf *g, int index, char *name, size_t name_cap, int *type,
                                       int *rank, int64_t *dims, int64_t *offset, int64_t *bytes)
{
    if (!g) return set_error(SATORI_ERR_DISPOSED, "GGUF file is closed");
    if (index < 0 || index >= (int)g->tensors.size()) return set_error(SATORI_ERR_ARGUMENT, "tensor index %d", index);
    const TensorRec &t = g->tensors[index];
    if (name && name_cap) {
        const size_t n = std::min(name_cap - 1, t.name.size());
        memcpy(name, t.name.data(), n);
        name[n] = 0;
    }
    if (type) *type = (int)t.type;
    if (rank) *rank = t.rank;
    if (dims)
        for (int d = 0; d < 4; ++d) dims[d] = d < t.rank ? t.dims[d] : 1;
    if (offset) *offset = t.offset;
    if (bytes) *bytes = t.bytes;
    return SATORI_OK;
}

extern "C" int satori_gguf_find_tensor(const satori_gguf *g, const char *name, int *index)
{
    if (!g) return set_error(SATORI_ERR_DISPOSED, "GGUF file is closed");
    if (!name || !index) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    auto it = g->tensor_index.find(name);
    *index = it == g->tensor_index.end() ? -1 : (int)it->second;
    return SATORI_OK;
}

extern "C" const void *satori_gguf_tensor_data(const satori_gguf *g, int index)
{
    if (!g || index < 0 || index >= (int)g->tensors.size()) return nullptr;
    return g->map + g->tensors[index].offset;
}

extern "C" int satori_gguf_metadata(const satori_gguf *g, int index, char *key, size_t key_cap, int *type,
                                    int *elem_type, int64_t *count)
{
    if (!g) return set_error(SATORI_ERR_DISPOSED, "GGUF file is closed");
    if (index < 0 || index >= (int)g->meta.size()) return set_error(SATORI_ERR_ARGUMENT, "metadata index %d", index);
    const Meta &m = g->meta[index];
    if (key && key_cap) {
        const size_t n = std::min(key_cap - 1, m.key.size());
        memcpy(key, m.key.data(), n);
        key[n] = 0;
    }
    if (type) *type = (int)m.type;
    if (elem_type) *elem_type = m.type == 9 ? (int)m.elem_type : -1;
    if (count) *count = m.type == 9 ? m.count : 1;
    return SATORI_OK;
}

extern "C" int satori_gguf_read_scalar(const satori_gguf *g, const char *key, int *type, void *out, size_t cap,
                                       size_t *written)
{
    if (!g) return set_error(SATORI_ERR_DISPOSED, "GGUF file is closed");
    if (!key) return set_error(SATORI_ERR_ARGUMENT, "null key");
    const Meta *m = g->find_meta(key);
    if (!m) return set_error(SATORI_ERR_ARGUMENT, "no metadata key %s", key);
    // GgufFile.ReadScalar (GgufFile.cs:56-76): arrays need scoped access.
    if (m->type == 9) return set_error(SATORI_ERR_ARGUMENT, "Use scoped access for arrays.");
    if (type) *type = (int)m->type;
    const uint8_t *src = g->map + m->offset + (m->type == 8 ? 8 : 0);
    const size_t n = (size_t)(m->type == 8 ? m->length - 8 : m->length);
    if (written) *written = n;
    if (out) {
        if (cap < n) return set_error(SATORI_ERR_ARGUMENT, "buffer of %zu bytes is smaller than %zu", cap, n);
        memcpy(out, src, n);
    }
    return SATORI_OK;
}

// Fills a model description from the file: DenseTransformerAdapter.Validate over ModelConfig, then one
// satori_tensor per tensor the session reads (host pointers into the mapping).
extern "C" int satori_gguf_model_desc(const satori_gguf *g, satori_model_desc *desc, satori_tensor *tensors,
                                      int capacity, int *needed)
{
    if (!g) return set_error(SATORI_ERR_DISPOSED, "GGUF file is closed");
    if (!desc) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    const std::string a = g->architecture;
    if (a != "qwen2" && a != "qwen3")
        return set_error(SATORI_ERR_NOT_SUPPORTED, "architecture %s: only qwen2 and qwen3 dense decoders", a.c_str());
    auto key = [&](const char *suffix) { return a + "." + suffix; };
    int64_t layers, embedding, ffn, heads, heads_kv;
    double eps, rope;
    std::string gaps;
    auto gap = [&](const char *what, const char *why) {
        gaps += std::string(gaps.empty() ? "" : "; ") + what + ": " + why;
    };
    if (!meta_int(g, key("block_count"), &layers) || layers <= 0) gap("block_count", "missing or non-positive");
    if (!meta_int(g, key("embedding_length"), &embedding) || embedding <= 0)
        gap("embedding_length", "missing or non-positive");
    if (!meta_int(g, key("feed_forward_length"), &ffn) || ffn <= 0) gap("feed_forward_length", "missing or non-positive");
    if (!meta_int(g, key("attention.head_count"), &heads) || heads <= 0)
        gap("attention.head_count", "missing or non-positive");
    if (!meta_int(g, key("attention.head_count_kv"), &heads_kv) || heads_kv <= 0)
        gap("attention.head_count_kv", "missing or non-positive");
    if (!meta_float(g, key("attention.layer_norm_rms_epsilon"), &eps) || !(eps > 0))
        gap("attention.layer_norm_rms_epsilon", "missing or non-positive");
    if (!meta_float(g, key("rope.freq_base"), &rope) || !(rope > 0)) gap("rope.freq_base", "missing or non-positive");
    if (!gaps.empty()) return set_error(SATORI_ERR_NOT_SUPPORTED, "capability gaps: %s", gaps.c_str());
    if (heads_kv > heads) return set_error(SATORI_ERR_NOT_SUPPORTED, "attention.head_count_kv greater than head_count");
    if (layers > INT32_MAX || embedding > INT32_MAX || ffn > INT32_MAX || heads > INT32_MAX)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "a derived dimension exceeds Int32");
    int64_t head_dim;
    int64_t key_length;
    if (meta_int(g, key("attention.key_length"), &key_length)) {
        if (key_length <= 0 || key_length > INT32_MAX)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "attention.key_length non-positive or exceeds Int32");
        head_dim = key_length;
    } else {
        if (embedding % heads != 0)
            return set_error(SATORI_ERR_NOT_SUPPORTED, "attention.key_length absent and embedding_length %lld is not "
                             "divisible by head_count %lld", (long long)embedding, (long long)heads);
        head_dim = embedding / heads;
    }
    int64_t vocab = -1, declared;
    const TensorRec *embd = tensor(g, "token_embd.weight");
    if (meta_int(g, key("vocab_size"), &declared) && declared > 0) vocab = declared > INT32_MAX ? -1 : declared;
    else if (embd && embd->rank == 2) vocab = embd->dims[1];
    if (vocab <= 0) return set_error(SATORI_ERR_NOT_SUPPORTED, "vocab_size not declared and not derivable");
    const int64_t q_width = heads * head_dim, kv_width = heads_kv * head_dim;
    if (q_width > INT32_MAX || kv_width > INT32_MAX)
        return set_error(SATORI_ERR_NOT_SUPPORTED, "attention.key_length: a derived width exceeds Int32");
    const bool has_output = tensor(g, "output.weight") != nullptr;
    bool tied_flag = false;
    const bool tied = (meta_bool(g, key("tie_word_embeddings"), &tied_flag) && tied_flag) || !has_output;

    // Required tensors with their GGUF dimensions [cols, rows] (vectors: [n]).
    struct Want {
        std::string name;
        int64_t d0, d1;   // d1 = 0: a vector
        bool optional;
    };
    std::vector<Want> want;
    want.push_back({"token_embd.weight", embedding, vocab, false});
    want.push_back({"output_norm.weight", embedding, 0, false});
    if (has_output && !tied) want.push_back({"output.weight", embedding, vocab, false});
    for (int64_t l = 0; l < layers; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        want.push_back({p + "attn_norm.weight", embedding, 0, false});
        want.push_back({p + "attn_q.weight", embedding, q_width, false});
        want.push_back({p + "attn_k.weight", embedding, kv_width, false});
        want.push_back({p + "attn_v.weight", embedding, kv_width, false});
        want.push_back({p + "attn_output.weight", q_width, embedding, false});
        want.push_back({p + "ffn_norm.weight", embedding, 0, false});
        want.push_back({p + "ffn_gate.weight", embedding, ffn, false});
        want.push_back({p + "ffn_up.weight", embedding, ffn, false});
        want.push_back({p + "ffn_down.weight", ffn, embedding, false});
        want.push_back({p + "attn_q.bias", q_width, 0, true});
        want.push_back({p + "attn_k.bias", kv_width, 0, true});
        want.push_back({p + "attn_v.bias", kv_width, 0, true});
        want.push_back({p + "attn_q_norm.weight", head_dim, 0, true});
        want.push_back({p + "attn_k_norm.weight", head_dim, 0, true});
    }
    int n = 0;
    for (const Want &w : want) {
        const TensorRec *t = tensor(g, w.name);
        if (!t) {
            if (w.optional) continue;
            return set_error(SATORI_ERR_NOT_SUPPORTED, "missing tensor %s", w.name.c_str());
        }
        const bool matrix = w.d1 != 0;
        if (t->rank != (matrix ? 2 : 1) || t->dims[0] != w.d0 || (matrix && t->dims[1] != w.d1))
            return set_error(SATORI_ERR_NOT_SUPPORTED, "tensor %s has an unexpected shape", w.name.c_str());
        int format;
        if (matrix) {
            if (t->type == 8) format = SATORI_Q8_0;
            else if (t->type == 2) format = SATORI_Q4_0;
            else if (t->type == 12) format = SATORI_Q4_K;
            else if (t->type == 14) format = SATORI_Q6_K;
            else return set_error(SATORI_ERR_NOT_SUPPORTED, "tensor %s: GGUF type %u is not a supported matrix format",
                                  w.name.c_str(), t->type);
        } else {
            if (t->type != 0)
                return set_error(SATORI_ERR_NOT_SUPPORTED, "tensor %s: vectors must be F32", w.name.c_str());
            format = -1;
        }
        if (tensors && n < capacity) {
            satori_tensor &o = tensors[n];
            o.name = t->name.c_str();
            o.data = g->map + t->offset;
            o.bytes = (size_t)t->bytes;
            o.format = format;
            o.rows = matrix ? (int)t->dims[1] : (int)t->dims[0];
            o.cols = matrix ? (int)t->dims[0] : 1;
        }
        ++n;
    }
    if (needed) *needed = n;
    desc->layers = (int)layers;
    desc->hidden = (int)embedding;
    desc->ffn = (int)ffn;
    desc->q_heads = (int)heads;
    desc->kv_heads = (int)heads_kv;
    desc->head_dim = (int)head_dim;
    desc->vocab = (int)vocab;
    desc->rms_epsilon = (float)eps;
    desc->rope_base = rope;
    desc->tied_embeddings = tied ? 1 : 0;
    desc->n_tensors = std::min(n, capacity);
    desc->tensors = tensors;
    if (tensors && capacity < n) return set_error(SATORI_ERR_ARGUMENT, "tensor table needs %d entries", n);
    return SATORI_OK;
}

extern "C" int satori_session_create_from_gguf(satori_ctx *ctx, const satori_gguf *g, int context, satori_session **out)
{
    if (!g) return set_error(SATORI_ERR_DISPOSED, "GGUF file is closed");
    satori_model_desc d = {};
    int needed = 0;
    int rc = satori_gguf_model_desc(g, &d, nullptr, 0, &needed);
    if (rc) return rc;
    std::vector<satori_tensor> table((size_t)needed);
    rc = satori_gguf_model_desc(g, &d, table.data(), needed, &needed);
    if (rc) return rc;
    return satori_session_create(ctx, &d, context, out);
}

// ---------------------------------------------------------------------------------------- STQ2
// MappedTernary2Matrix (src/Satori.Core/MappedTernary2Matrix.cs:9-30) with the header rules of
// Ternary2FileFormat.ReadHeader (src/Satori.Core/Ternary2FileFormat.cs:21-35): the file is mapped, the
// header and the total length checked, the payload validated and uploaded once.
extern "C" int satori_stq2_open(satori_ctx *ctx, const char *path, satori_matrix **out)
{
    if (!ctx || !path || !out) return set_error(SATORI_ERR_ARGUMENT, "null argument");
    int fd = -1;
    const uint8_t *map = nullptr;
    int64_t len = 0;
    int rc = map_file(path, INT64_MAX, &fd, &map, &len);
    if (rc) return rc;
    auto done = [&](int status) {
        if (map) munmap(const_cast<uint8_t *>(map), (size_t)len);
        close(fd);
        return status;
    };
    if (len < 32) return done(set_error(SATORI_ERR_INVALID_DATA, "Truncated Ternary2 header."));
    auto rd32 = [&](int o) {
        int32_t v;
        memcpy(&v, map + o, 4);
        return v;
    };
    uint16_t version, header;
    memcpy(&version, map + 4, 2);
    memcpy(&header, map + 6, 2);
    if (memcmp(map, "STQ2", 4) != 0 || version != 1 || header != 32 || rd32(20) != 0)
        return done(set_error(SATORI_ERR_INVALID_DATA, "Unsupported Ternary2 header."));
    const int rows = rd32(8), cols = rd32(12), bs = rd32(16);
    // Ternary2Shape (Ternary2Shape.cs:5-22); a bad shape is an InvalidDataException when mapped.
    if (rows <= 0 || cols <= 0 || (bs != 64 && bs != 128 && bs != 256))
        return done(set_error(SATORI_ERR_INVALID_DATA, "Invalid Ternary2 shape or payload."));
    const int64_t bpr = ((int64_t)cols + bs - 1) / bs;
    const int64_t payload = (int64_t)rows * bpr * (4 + bs / 4);
    if (payload > INT32_MAX) return done(set_error(SATORI_ERR_INVALID_DATA, "Invalid Ternary2 shape or payload."));
    int64_t declared;
    memcpy(&declared, map + 24, 8);
    if (declared != payload) return done(set_error(SATORI_ERR_INVALID_DATA, "Payload length disagrees with matrix shape."));
    if (len != 32 + payload) return done(set_error(SATORI_ERR_INVALID_DATA, "Truncated payload or trailing file data."));
    rc = satori_matrix_create(ctx, map + 32, (size_t)payload, rows, cols, bs, out);
    // Ternary2Matrix.ValidatePayload's ArgumentException becomes InvalidDataException for a mapped file.
    if (rc == SATORI_ERR_ARGUMENT) rc = SATORI_ERR_INVALID_DATA;
    return done(rc);
}
