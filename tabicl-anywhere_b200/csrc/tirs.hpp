// The `.tirs` tensor bundle, read and written byte-compatibly with tabicl-anywhere (src/store.rs:1-11,
// 282-483): magic "TIRSBNDL", u64 index length, a text index "name dtype offset nbytes dims...", tensors on
// 64-byte boundaries. Reads copy ranges into caller buffers (no mapping), as store.rs does.
#pragma once
#include <cstdint>
#include <cstdio>
#include <functional>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace tcu {

struct BundleError : std::runtime_error {
    int code;
    BundleError(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};

struct Entry {
    std::string name, dtype;
    uint64_t offset = 0, nbytes = 0;
    std::vector<uint64_t> dims;
    uint64_t len() const;
};

// store.rs:190-199 f16_to_f32: exact widening of IEEE binary16
float f16_to_f32(uint16_t h);
// store.rs:203-225 f32_to_f16: nearest, ties to even, overflow to the largest finite value
uint16_t f32_to_f16(float x);
int dtype_size(const std::string &d);

// store.rs:282-413 Bundle (file-backed or in-memory source)
class Bundle {
  public:
    static std::unique_ptr<Bundle> open(const std::string &path);
    static std::unique_ptr<Bundle> from_bytes(std::vector<uint8_t> bytes);
    // A source read by the caller's positional reads (store.rs:45-50 ReadAt: a file, memory, object storage, a
    // sealed bundle decrypted as it is read): read(buf, n, offset) fills buf or throws BundleError.
    static std::unique_ptr<Bundle> from_reader(std::function<void(void *, uint64_t, uint64_t)> read, uint64_t size);
    ~Bundle();
    bool has(const std::string &name) const { return by_name_.count(name) != 0; }
    const Entry &entry(const std::string &name) const;
    // store.rs:363-380: float32, or float16 widened on read
    void read_f32_at(const std::string &name, uint64_t skip, float *out, uint64_t count) const;
    std::vector<float> f32s(const std::string &name) const;
    std::vector<int32_t> i32s(const std::string &name) const;
    // store.rs:383-389
    void read_bytes_at(const std::string &name, uint64_t skip, void *out, uint64_t count) const;
    std::vector<uint8_t> bytes(const std::string &name) const;
    const std::vector<Entry> &entries() const { return entries_; }

  private:
    Bundle() = default;
    void parse();
    void read_at(void *buf, uint64_t n, uint64_t offset) const;
    FILE *file_ = nullptr;
    std::vector<uint8_t> mem_;
    std::function<void(void *, uint64_t, uint64_t)> reader_;
    uint64_t size_ = 0;
    std::vector<Entry> entries_;
    std::map<std::string, size_t> by_name_;
};

// store.rs:417-483 BundleWriter: all shapes known up front, data filled in any order
class BundleWriter {
  public:
    struct Spec {
        std::string name, dtype;
        std::vector<uint64_t> dims;
    };
    BundleWriter(const std::string &path, const std::vector<Spec> &tensors);
    ~BundleWriter();
    void write_bytes_at(const std::string &name, uint64_t skip, const void *data, uint64_t n);
    const Entry &entry(const std::string &name) const;

  private:
    FILE *file_ = nullptr;
    std::vector<Entry> entries_;
    std::map<std::string, size_t> by_name_;
};

}  // namespace tcu
