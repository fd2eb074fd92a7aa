// JSON and ZIP readers for .armpack packages (see sdk_io.h).
#include "sdk_io.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <zlib.h>

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <cstring>
#include <dirent.h>
#include <functional>

namespace sgsdk {

// ================================================================== JSON
namespace {

const Json kNull{};

struct Parser {
  const std::string& s;
  size_t i = 0;
  std::string err;

  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool fail(const char* what) {
    if (err.empty()) err = std::string(what) + " at offset " + std::to_string(i);
    return false;
  }
  bool lit(const char* w) {
    const size_t n = strlen(w);
    if (s.compare(i, n, w) != 0) return false;
    i += n;
    return true;
  }
  static void put_utf8(std::string& o, uint32_t cp) {
    if (cp < 0x80) {
      o += (char)cp;
    } else if (cp < 0x800) {
      o += (char)(0xC0 | (cp >> 6));
      o += (char)(0x80 | (cp & 0x3F));
    } else if (cp < 0x10000) {
      o += (char)(0xE0 | (cp >> 12));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    } else {
      o += (char)(0xF0 | (cp >> 18));
      o += (char)(0x80 | ((cp >> 12) & 0x3F));
      o += (char)(0x80 | ((cp >> 6) & 0x3F));
      o += (char)(0x80 | (cp & 0x3F));
    }
  }
  bool hex4(uint32_t* v) {
    if (i + 4 > s.size()) return fail("truncated \\u escape");
    *v = 0;
    for (int k = 0; k < 4; ++k) {
      const char c = s[i++];
      *v <<= 4;
      if (c >= '0' && c <= '9') *v |= (uint32_t)(c - '0');
      else if (c >= 'a' && c <= 'f') *v |= (uint32_t)(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') *v |= (uint32_t)(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    return true;
  }
  bool string(std::string* out) {
    if (i >= s.size() || s[i] != '"') return fail("expected string");
    ++i;
    out->clear();
    while (i < s.size()) {
      const char c = s[i++];
      if (c == '"') return true;
      if (c != '\\') {
        *out += c;
        continue;
      }
      if (i >= s.size()) break;
      const char e = s[i++];
      switch (e) {
        case '"': *out += '"'; break;
        case '\\': *out += '\\'; break;
        case '/': *out += '/'; break;
        case 'b': *out += '\b'; break;
        case 'f': *out += '\f'; break;
        case 'n': *out += '\n'; break;
        case 'r': *out += '\r'; break;
        case 't': *out += '\t'; break;
        case 'u': {
          uint32_t cp = 0;
          if (!hex4(&cp)) return false;
          if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' && s[i + 1] == 'u') {
            i += 2;
            uint32_t lo = 0;
            if (!hex4(&lo)) return false;
            cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
          }
          put_utf8(*out, cp);
          break;
        }
        default: return fail("bad escape");
      }
    }
    return fail("unterminated string");
  }
  bool value(Json* v, int depth) {
    if (depth > 200) return fail("nesting too deep");
    ws();
    if (i >= s.size()) return fail("unexpected end");
    const char c = s[i];
    if (c == '{') {
      v->kind = Json::Object;
      ++i;
      ws();
      if (i < s.size() && s[i] == '}') {
        ++i;
        return true;
      }
      for (;;) {
        ws();
        std::string k;
        if (!string(&k)) return false;
        ws();
        if (i >= s.size() || s[i] != ':') return fail("expected ':'");
        ++i;
        Json child;
        if (!value(&child, depth + 1)) return false;
        v->obj[k] = std::move(child);
        ws();
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == '}') {
          ++i;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      v->kind = Json::Array;
      ++i;
      ws();
      if (i < s.size() && s[i] == ']') {
        ++i;
        return true;
      }
      for (;;) {
        Json child;
        if (!value(&child, depth + 1)) return false;
        v->arr.push_back(std::move(child));
        ws();
        if (i < s.size() && s[i] == ',') {
          ++i;
          continue;
        }
        if (i < s.size() && s[i] == ']') {
          ++i;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v->kind = Json::String;
      return string(&v->str);
    }
    if (lit("true")) {
      v->kind = Json::Bool;
      v->b = true;
      return true;
    }
    if (lit("false")) {
      v->kind = Json::Bool;
      v->b = false;
      return true;
    }
    if (lit("null")) {
      v->kind = Json::Null;
      return true;
    }
    // number
    const size_t start = i;
    if (i < s.size() && (s[i] == '-' || s[i] == '+')) ++i;
    while (i < s.size() && (isdigit((unsigned char)s[i]) || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                            s[i] == '-' || s[i] == '+'))
      ++i;
    if (i == start) return fail("unexpected character");
    char* end = nullptr;
    const std::string tok = s.substr(start, i - start);
    v->kind = Json::Number;
    v->num = strtod(tok.c_str(), &end);
    if (!end || *end != '\0') return fail("bad number");
    return true;
  }
};

}  // namespace

const Json& Json::operator[](const std::string& k) const {
  if (kind != Object) return kNull;
  auto it = obj.find(k);
  return it == obj.end() ? kNull : it->second;
}
const Json& Json::operator[](size_t i) const {
  if (kind != Array || i >= arr.size()) return kNull;
  return arr[i];
}

bool json_parse(const std::string& text, Json* out, std::string* err) {
  Parser p{text};
  *out = Json{};
  if (!p.value(out, 0)) {
    *err = p.err;
    return false;
  }
  p.ws();
  if (p.i != text.size()) {
    *err = "trailing characters at offset " + std::to_string(p.i);
    return false;
  }
  return true;
}

// ================================================================== ZIP / directory
namespace {
uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }
uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

bool map_file(const std::string& path, int* fd_out, const uint8_t** p, uint64_t* n, std::string* err) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    *err = "cannot open " + path + ": " + strerror(errno);
    return false;
  }
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    *err = "cannot stat " + path;
    ::close(fd);
    return false;
  }
  *n = (uint64_t)st.st_size;
  if (*n == 0) {
    *p = nullptr;
    *fd_out = fd;
    return true;
  }
  void* m = mmap(nullptr, *n, PROT_READ, MAP_PRIVATE, fd, 0);
  if (m == MAP_FAILED) {
    *err = "cannot map " + path + ": " + strerror(errno);
    ::close(fd);
    return false;
  }
  *p = static_cast<const uint8_t*>(m);
  *fd_out = fd;
  return true;
}
}  // namespace

Container::~Container() {
  if (map_) munmap(const_cast<uint8_t*>(map_), map_size_);
  if (fd_ >= 0) ::close(fd_);
  for (auto& kv : file_maps_) {
    if (kv.second.p) munmap(const_cast<uint8_t*>(kv.second.p), kv.second.n);
    if (kv.second.fd >= 0) ::close(kv.second.fd);
  }
}

bool Container::open(const std::string& path, std::string* err) {
  struct stat st {};
  if (stat(path.c_str(), &st) != 0) {
    *err = "package not found: " + path;
    return false;
  }
  if (S_ISDIR(st.st_mode)) {
    is_dir_ = true;
    root_ = path;
    if (!root_.empty() && root_.back() != '/') root_ += '/';
    return true;
  }
  if (!map_file(path, &fd_, &map_, &map_size_, err)) return false;
  // End of central directory: last 22 + comment bytes.
  if (map_size_ < 22) {
    *err = "not a ZIP archive (too short): " + path;
    return false;
  }
  int64_t eocd = -1;
  const uint64_t lo = map_size_ > 65557 ? map_size_ - 65557 : 0;
  for (int64_t o = (int64_t)map_size_ - 22; o >= (int64_t)lo; --o)
    if (rd32(map_ + o) == 0x06054b50u) {
      eocd = o;
      break;
    }
  if (eocd < 0) {
    *err = "not a ZIP archive (no end-of-central-directory record): " + path;
    return false;
  }
  uint64_t n_entries = rd16(map_ + eocd + 10);
  uint64_t cd_size = rd32(map_ + eocd + 12);
  uint64_t cd_off = rd32(map_ + eocd + 16);
  // ZIP64 end-of-central-directory locator just before the EOCD.
  if ((cd_off == 0xFFFFFFFFu || n_entries == 0xFFFF) && eocd >= 20 && rd32(map_ + eocd - 20) == 0x07064b50u) {
    const uint64_t z64 = rd64(map_ + eocd - 20 + 8);
    if (z64 + 56 <= map_size_ && rd32(map_ + z64) == 0x06064b50u) {
      n_entries = rd64(map_ + z64 + 32);
      cd_size = rd64(map_ + z64 + 40);
      cd_off = rd64(map_ + z64 + 48);
    }
  }
  if (cd_off + cd_size > map_size_) {
    *err = "corrupt ZIP central directory: " + path;
    return false;
  }
  uint64_t o = cd_off;
  for (uint64_t k = 0; k < n_entries; ++k) {
    if (o + 46 > map_size_ || rd32(map_ + o) != 0x02014b50u) {
      *err = "corrupt ZIP central directory entry: " + path;
      return false;
    }
    Entry e;
    e.method = rd16(map_ + o + 10);
    e.csize = rd32(map_ + o + 20);
    e.usize = rd32(map_ + o + 24);
    const uint16_t nlen = rd16(map_ + o + 28), xlen = rd16(map_ + o + 30), clen = rd16(map_ + o + 32);
    e.local_offset = rd32(map_ + o + 42);
    if (o + 46 + nlen + xlen > map_size_) {
      *err = "corrupt ZIP entry name: " + path;
      return false;
    }
    const std::string name(reinterpret_cast<const char*>(map_ + o + 46), nlen);
    // ZIP64 extra field: the 0xFFFFFFFF sizes/offset follow in that order.
    const uint8_t* x = map_ + o + 46 + nlen;
    for (uint32_t xo = 0; xo + 4 <= xlen;) {
      const uint16_t id = rd16(x + xo), sz = rd16(x + xo + 2);
      if (id == 0x0001) {
        uint32_t q = xo + 4;
        if (e.usize == 0xFFFFFFFFu && q + 8 <= xo + 4u + sz) { e.usize = rd64(x + q); q += 8; }
        if (e.csize == 0xFFFFFFFFu && q + 8 <= xo + 4u + sz) { e.csize = rd64(x + q); q += 8; }
        if (e.local_offset == 0xFFFFFFFFu && q + 8 <= xo + 4u + sz) { e.local_offset = rd64(x + q); q += 8; }
      }
      xo += 4u + sz;
    }
    entries_[name] = e;
    o += 46 + nlen + xlen + clen;
  }
  return true;
}

bool Container::exists(const std::string& name) const {
  if (is_dir_) {
    struct stat st {};
    return stat((root_ + name).c_str(), &st) == 0;
  }
  return entries_.count(name) != 0;
}

std::vector<std::string> Container::names() const {
  std::vector<std::string> out;
  if (is_dir_) {
    std::function<void(const std::string&)> walk = [&](const std::string& rel) {
      DIR* d = opendir((root_ + rel).c_str());
      if (!d) return;
      while (dirent* de = readdir(d)) {
        const std::string n = de->d_name;
        if (n == "." || n == "..") continue;
        const std::string r = rel + n;
        struct stat st {};
        if (stat((root_ + r).c_str(), &st) == 0 && S_ISDIR(st.st_mode)) walk(r + "/");
        else out.push_back(r);
      }
      closedir(d);
    };
    walk("");
  } else {
    for (auto& kv : entries_) out.push_back(kv.first);
  }
  return out;
}

bool Container::entry_data(const Entry& e, const uint8_t** p, std::string* err) const {
  if (e.local_offset + 30 > map_size_ || rd32(map_ + e.local_offset) != 0x04034b50u) {
    *err = "corrupt ZIP local header";
    return false;
  }
  const uint16_t nlen = rd16(map_ + e.local_offset + 26), xlen = rd16(map_ + e.local_offset + 28);
  const uint64_t start = e.local_offset + 30 + nlen + xlen;
  if (start + e.csize > map_size_) {
    *err = "truncated ZIP entry";
    return false;
  }
  *p = map_ + start;
  return true;
}

bool Container::map_entry(const std::string& name, const uint8_t** data, uint64_t* size, std::string* err) {
  if (is_dir_) {
    auto it = file_maps_.find(name);
    if (it == file_maps_.end()) {
      FileMap fm;
      if (!map_file(root_ + name, &fm.fd, &fm.p, &fm.n, err)) return false;
      it = file_maps_.emplace(name, fm).first;
    }
    *data = it->second.p;
    *size = it->second.n;
    return true;
  }
  auto it = entries_.find(name);
  if (it == entries_.end()) {
    *err = "entry not in package: " + name;
    return false;
  }
  const Entry& e = it->second;
  const uint8_t* p = nullptr;
  if (!entry_data(e, &p, err)) return false;
  if (e.method == 0) {
    *data = p;
    *size = e.usize;
    return true;
  }
  if (e.method != 8) {
    *err = "unsupported ZIP compression method " + std::to_string(e.method) + " for " + name;
    return false;
  }
  auto inf = inflated_.find(name);
  if (inf == inflated_.end()) {
    auto buf = std::make_unique<std::vector<uint8_t>>(e.usize);
    z_stream zs{};
    if (inflateInit2(&zs, -MAX_WBITS) != Z_OK) {
      *err = "inflateInit failed";
      return false;
    }
    uint64_t in_left = e.csize, out_done = 0;
    const uint8_t* in = p;
    int rc = Z_OK;
    while (rc != Z_STREAM_END) {
      const uInt in_chunk = (uInt)std::min<uint64_t>(in_left, 1u << 30);
      const uInt out_chunk = (uInt)std::min<uint64_t>(e.usize - out_done, 1u << 30);
      zs.next_in = const_cast<Bytef*>(in);
      zs.avail_in = in_chunk;
      zs.next_out = buf->data() + out_done;
      zs.avail_out = out_chunk;
      rc = inflate(&zs, Z_NO_FLUSH);
      const uint64_t used_in = in_chunk - zs.avail_in, made = out_chunk - zs.avail_out;
      in += used_in;
      in_left -= used_in;
      out_done += made;
      if (rc != Z_OK && rc != Z_STREAM_END) break;
      if (used_in == 0 && made == 0) break;
    }
    inflateEnd(&zs);
    if (rc != Z_STREAM_END || out_done != e.usize) {
      *err = "corrupt deflated entry " + name;
      return false;
    }
    inf = inflated_.emplace(name, std::move(buf)).first;
  }
  *data = inf->second->data();
  *size = inf->second->size();
  return true;
}

bool Container::read_text(const std::string& name, std::string* out, std::string* err) const {
  Container* self = const_cast<Container*>(this);
  const uint8_t* p = nullptr;
  uint64_t n = 0;
  if (!self->map_entry(name, &p, &n, err)) return false;
  out->assign(reinterpret_cast<const char*>(p), n);
  return true;
}

}  // namespace sgsdk
