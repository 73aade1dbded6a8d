// `.tirs` bundle reader and writer (src/store.rs:1-11, 190-225, 282-483 of tabicl-anywhere).
#include "tirs.hpp"

#include "../../include/tabicl_b200.h"

#include <cstring>
#include <sstream>

namespace tcu {

static const char MAGIC[8] = {'T', 'I', 'R', 'S', 'B', 'N', 'D', 'L'};
static const uint64_t MAX_INDEX = 64ull << 20;  // store.rs:23

uint64_t Entry::len() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
}

int dtype_size(const std::string &d) {
    if (d == "float32" || d == "int32") return 4;
    if (d == "float16") return 2;
    if (d == "uint8" || d == "int8") return 1;
    if (d == "float64" || d == "int64") return 8;
    return 0;
}

float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        // zero and subnormals: man * 2^-24, exact in 32 bits
        float v = (float)man * (1.0f / 16777216.0f);
        std::memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

uint16_t f32_to_f16(float x) {
    uint32_t b;
    std::memcpy(&b, &x, 4);
    uint16_t sign = (uint16_t)((b >> 16) & 0x8000);
    int32_t exp = (int32_t)((b >> 23) & 0xff);
    uint32_t man = b & 0x7fffff;
    if (exp == 255) return sign | (man != 0 ? 0x7e00 : 0x7bff);
    int32_t e = exp - 112;
    if (e >= 31) return sign | 0x7bff;
    auto nearest = [](uint32_t kept, uint32_t rest, uint32_t half) {
        return kept + (uint32_t)(rest > half || (rest == half && (kept & 1)));
    };
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t m = man | 0x800000, shift = (uint32_t)(14 - e);
        return sign | (uint16_t)nearest(m >> shift, m & ((1u << shift) - 1), 1u << (shift - 1));
    }
    uint32_t v = nearest(((uint32_t)e << 10) | (man >> 13), man & 0x1fff, 0x1000);
    return sign | (uint16_t)(v < 0x7bff ? v : 0x7bff);
}

std::unique_ptr<Bundle> Bundle::open(const std::string &path) {
    std::unique_ptr<Bundle> b(new Bundle());
    b->file_ = std::fopen(path.c_str(), "rb");
    if (!b->file_) throw BundleError(TCU_ERR_IO, path + ": cannot open");
    std::fseek(b->file_, 0, SEEK_END);
    b->size_ = (uint64_t)std::ftell(b->file_);
    try {
        b->parse();
    } catch (BundleError &e) {
        throw BundleError(e.code, path + ": " + e.what());
    }
    return b;
}

std::unique_ptr<Bundle> Bundle::from_bytes(std::vector<uint8_t> bytes) {
    std::unique_ptr<Bundle> b(new Bundle());
    b->mem_ = std::move(bytes);
    b->size_ = b->mem_.size();
    b->parse();
    return b;
}

std::unique_ptr<Bundle> Bundle::from_reader(std::function<void(void *, uint64_t, uint64_t)> read, uint64_t size) {
    std::unique_ptr<Bundle> b(new Bundle());
    b->reader_ = std::move(read);
    b->size_ = size;
    b->parse();
    return b;
}

Bundle::~Bundle() {
    if (file_) std::fclose(file_);
}

void Bundle::read_at(void *buf, uint64_t n, uint64_t offset) const {
    if (offset > size_ || n > size_ - offset) throw BundleError(TCU_ERR_FORMAT, "read past the end of the bundle");
    if (reader_) {
        reader_(buf, n, offset);
        return;
    }
    if (!file_) {
        std::memcpy(buf, mem_.data() + offset, n);
        return;
    }
    if (std::fseek(file_, (long)offset, SEEK_SET) != 0 || std::fread(buf, 1, n, file_) != n)
        throw BundleError(TCU_ERR_IO, "short read");
}

// store.rs:316-351 from_source: header, then index, each line's shape checked against its byte count
void Bundle::parse() {
    uint8_t head[16];
    read_at(head, 16, 0);
    if (std::memcmp(head, MAGIC, 8) != 0) throw BundleError(TCU_ERR_FORMAT, "not a tabicl-anywhere bundle");
    uint64_t index_len;
    std::memcpy(&index_len, head + 8, 8);
    if (index_len > MAX_INDEX) throw BundleError(TCU_ERR_FORMAT, "bundle index too large; the file is damaged");
    std::string text(index_len, '\0');
    read_at(&text[0], index_len, 16);
    std::istringstream lines(text);
    std::string line;
    while (std::getline(lines, line)) {
        if (line.empty()) continue;
        std::istringstream f(line);
        Entry e;
        if (!(f >> e.name >> e.dtype >> e.offset >> e.nbytes)) throw BundleError(TCU_ERR_FORMAT, "short index line: " + line);
        uint64_t v;
        while (f >> v) e.dims.push_back(v);
        int w = dtype_size(e.dtype);
        if (!w) throw BundleError(TCU_ERR_FORMAT, line + ": unknown tensor type");
        if (e.len() * (uint64_t)w != e.nbytes) throw BundleError(TCU_ERR_FORMAT, line + ": shape and length disagree");
        by_name_[e.name] = entries_.size();
        entries_.push_back(e);
    }
}

const Entry &Bundle::entry(const std::string &name) const {
    auto it = by_name_.find(name);
    if (it == by_name_.end()) throw BundleError(TCU_ERR_FORMAT, "bundle has no tensor named " + name);
    return entries_[it->second];
}

void Bundle::read_f32_at(const std::string &name, uint64_t skip, float *out, uint64_t count) const {
    const Entry &e = entry(name);
    if (e.dtype == "float16") {
        if ((skip + count) * 2 > e.nbytes) throw BundleError(TCU_ERR_FORMAT, name + ": read past the end");
        std::vector<uint16_t> raw(count);
        read_at(raw.data(), count * 2, e.offset + 2 * skip);
        for (uint64_t i = 0; i < count; i++) out[i] = f16_to_f32(raw[i]);
        return;
    }
    if (e.dtype != "float32" || (skip + count) * 4 > e.nbytes)
        throw BundleError(TCU_ERR_FORMAT, name + ": not float32 or read past the end");
    read_at(out, count * 4, e.offset + 4 * skip);
}

std::vector<float> Bundle::f32s(const std::string &name) const {
    std::vector<float> v(entry(name).len());
    read_f32_at(name, 0, v.data(), v.size());
    return v;
}

std::vector<int32_t> Bundle::i32s(const std::string &name) const {
    const Entry &e = entry(name);
    if (e.dtype != "int32") throw BundleError(TCU_ERR_FORMAT, name + ": is " + e.dtype + ", wanted int32");
    std::vector<int32_t> v(e.len());
    read_at(v.data(), e.nbytes, e.offset);
    return v;
}

void Bundle::read_bytes_at(const std::string &name, uint64_t skip, void *out, uint64_t count) const {
    const Entry &e = entry(name);
    if (skip + count > e.nbytes) throw BundleError(TCU_ERR_FORMAT, name + ": read past the end");
    read_at(out, count, e.offset + skip);
}

std::vector<uint8_t> Bundle::bytes(const std::string &name) const {
    const Entry &e = entry(name);
    std::vector<uint8_t> v(e.nbytes);
    read_at(v.data(), e.nbytes, e.offset);
    return v;
}

// store.rs:431-464 create_on: lay the index out with a generous offset width, tensors 64-byte aligned
BundleWriter::BundleWriter(const std::string &path, const std::vector<Spec> &tensors) {
    auto line = [](const Spec &s, uint64_t off, uint64_t nb) {
        std::string l = s.name + " " + s.dtype + " " + std::to_string(off) + " " + std::to_string(nb);
        for (auto v : s.dims) l += " " + std::to_string(v);
        return l + "\n";
    };
    std::vector<uint64_t> sizes;
    uint64_t guess = 0;
    for (auto &s : tensors) {
        if (s.name.empty() || s.name.find_first_of(" \n") != std::string::npos)
            throw BundleError(TCU_ERR_ARG, "tensor name '" + s.name + "' is empty or has a space or line break");
        int w = dtype_size(s.dtype);
        if (!w) throw BundleError(TCU_ERR_ARG, "unknown tensor type " + s.dtype);
        uint64_t n = 1;
        for (auto d : s.dims) n *= d;
        sizes.push_back(n * (uint64_t)w);
        guess += line(s, 1000000000000000ull, sizes.back()).size();
    }
    uint64_t pos = (guess + 16 + 63) / 64 * 64;
    std::string index;
    for (size_t i = 0; i < tensors.size(); i++) {
        index += line(tensors[i], pos, sizes[i]);
        Entry e;
        e.name = tensors[i].name, e.dtype = tensors[i].dtype, e.offset = pos, e.nbytes = sizes[i], e.dims = tensors[i].dims;
        by_name_[e.name] = entries_.size();
        entries_.push_back(e);
        pos = (pos + sizes[i] + 63) / 64 * 64;
    }
    file_ = std::fopen(path.c_str(), "w+b");
    if (!file_) throw BundleError(TCU_ERR_IO, path + ": cannot create");
    uint64_t len = index.size();
    std::fwrite(MAGIC, 1, 8, file_);
    std::fwrite(&len, 8, 1, file_);
    std::fwrite(index.data(), 1, index.size(), file_);
    // set the length: write a zero at the last byte
    if (pos > 0) {
        std::fseek(file_, (long)(pos - 1), SEEK_SET);
        std::fputc(0, file_);
    }
}

BundleWriter::~BundleWriter() {
    if (file_) std::fclose(file_);
}

const Entry &BundleWriter::entry(const std::string &name) const {
    auto it = by_name_.find(name);
    if (it == by_name_.end()) throw BundleError(TCU_ERR_ARG, "no tensor named " + name);
    return entries_[it->second];
}

void BundleWriter::write_bytes_at(const std::string &name, uint64_t skip, const void *data, uint64_t n) {
    const Entry &e = entry(name);
    if (skip + n > e.nbytes) throw BundleError(TCU_ERR_ARG, name + ": write past the end");
    std::fseek(file_, (long)(e.offset + skip), SEEK_SET);
    if (std::fwrite(data, 1, n, file_) != n) throw BundleError(TCU_ERR_IO, "short write");
}

}  // namespace tcu
