// Host-side readers for .armpack packages: a small JSON parser (manifest,
// graph and tensor-index files) and a ZIP reader (the package container,
// compiler/lib/package/package_generator.cpp:104-211 writes it with weights
// stored uncompressed so that they can be mapped in place).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace sgsdk {

// ------------------------------------------------------------------ JSON
struct Json {
  enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::map<std::string, Json> obj;

  bool has(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
  const Json& operator[](const std::string& k) const;  // Null value when absent
  const Json& operator[](size_t i) const;
  double number(double dflt = 0) const { return kind == Number ? num : (kind == Bool ? (b ? 1 : 0) : dflt); }
  int64_t integer(int64_t dflt = 0) const { return kind == Number ? (int64_t)num : dflt; }
  std::string text(const std::string& dflt = "") const { return kind == String ? str : dflt; }
  bool boolean(bool dflt = false) const { return kind == Bool ? b : (kind == Number ? num != 0 : dflt); }
  size_t size() const { return kind == Array ? arr.size() : (kind == Object ? obj.size() : 0); }
};

// Parses `text`; on a syntax error returns false and sets *err.
bool json_parse(const std::string& text, Json* out, std::string* err);

// ------------------------------------------------------------------ container
// A package is either a ZIP file or a directory with the same layout.
class Container {
 public:
  ~Container();
  // Opens `path`; false with *err on failure.
  bool open(const std::string& path, std::string* err);
  bool exists(const std::string& name) const;
  // Whole entry as text (inflates deflated ZIP entries).
  bool read_text(const std::string& name, std::string* out, std::string* err) const;
  // Pointer to an entry's bytes: in place for stored ZIP entries and files
  // (memory-mapped), else an inflated copy kept by the container.
  bool map_entry(const std::string& name, const uint8_t** data, uint64_t* size, std::string* err);
  std::vector<std::string> names() const;

 private:
  struct Entry {
    uint64_t local_offset = 0;
    uint64_t csize = 0, usize = 0;
    uint16_t method = 0;
  };
  bool is_dir_ = false;
  std::string root_;
  int fd_ = -1;
  const uint8_t* map_ = nullptr;
  uint64_t map_size_ = 0;
  std::map<std::string, Entry> entries_;
  std::map<std::string, std::unique_ptr<std::vector<uint8_t>>> inflated_;
  struct FileMap {
    int fd = -1;
    const uint8_t* p = nullptr;
    uint64_t n = 0;
  };
  std::map<std::string, FileMap> file_maps_;
  bool entry_data(const Entry& e, const uint8_t** p, std::string* err) const;
};

}  // namespace sgsdk
