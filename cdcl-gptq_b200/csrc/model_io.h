// model_io.h - safetensors files and the calibration-Hessian store on the host, for the model-level pipeline
// (the reference's src/io.rs: SafeTensors reading through mmap, write_tensors, HessianStore with aliases).
//
// Host C++ only; the dtype widening and the non-finite scan run on the device (io.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace cdclq {
namespace io {

// A JSON value: the subset safetensors headers and the `aliases` metadata use.
struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;  // insertion order kept
    const Json* get(const std::string& key) const;
};
// Parses one JSON document; false with a message in *err on malformed input.
bool parse_json(const char* s, size_t len, Json* out, std::string* err);
// `s` as a JSON string literal (quotes, escapes).
std::string json_quote(const std::string& s);

// Element size of a safetensors dtype name ("F32", "BF16", ...), 0 when unknown.
size_t dtype_size(const std::string& dtype);

struct TensorView {
    std::string dtype;
    std::vector<size_t> shape;
    const uint8_t* data = nullptr;
    size_t nbytes = 0;
    size_t numel() const {
        size_t n = 1;
        for (size_t d : shape) n *= d;
        return n;
    }
};

// A read-only, memory-mapped safetensors file (SafeTensors::deserialize over mmap_file, src/io.rs:25-30).
class SafeTensorsFile {
  public:
    SafeTensorsFile() = default;
    SafeTensorsFile(const SafeTensorsFile&) = delete;
    SafeTensorsFile& operator=(const SafeTensorsFile&) = delete;
    ~SafeTensorsFile();
    // 0, or CDCLQ_ERR_ARG with "<path>: <reason>" set as the library's last error.
    int open(const std::string& path);
    std::vector<std::string> names() const;  // sorted
    const TensorView* tensor(const std::string& name) const;
    const std::map<std::string, std::string>& metadata() const { return md_; }
    const std::string& path() const { return path_; }

  private:
    std::string path_;
    void* map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, TensorView> t_;
    std::map<std::string, std::string> md_;
};

// One tensor ready to be written (src/io.rs:90-95).
struct OutTensor {
    std::string name;
    std::string dtype;
    std::vector<size_t> shape;
    std::vector<uint8_t> bytes;
};

// write_tensors (src/io.rs:103-114): parent directories created; tensors laid out as the safetensors crate lays
// them out (larger dtypes first, then by name), the header padded with spaces to a multiple of 8 bytes.
int write_tensors(const std::string& path, const std::vector<OutTensor>& ts,
                  const std::map<std::string, std::string>& meta);

// HessianStore (src/io.rs:136-226): `<layer>.H` index over several files (later files override earlier ones),
// the `aliases` metadata ({layer: owner}) and square-shape checks.  The non-finite scan is the caller's (device).
class HessianStore {
  public:
    int open(const std::vector<std::string>& paths);
    // The layer whose `.H` serves `layer`: itself or its alias target (src/io.rs:172-182); "" when none.
    std::string resolve(const std::string& layer) const;
    // `<owner>.<suffix>` (suffix "H" or "M"): nullptr with *missing = true when the file has no such tensor;
    // nullptr with *missing = false and an error set when it is malformed (not square); else the view, n = side.
    const TensorView* tensor(const std::string& owner, const char* suffix, size_t* n, bool* missing) const;

  private:
    std::vector<std::unique_ptr<SafeTensorsFile>> files_;
    std::map<std::string, size_t> index_;
    std::map<std::string, std::string> aliases_;
};

}  // namespace io
}  // namespace cdclq
