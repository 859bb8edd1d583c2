// spt_gguf.cpp -- GGUF model index (see spt_gguf.h for the rules, which
// follow ggufindex.Open, ggufindex/index.go:55-575).
#include "spt_gguf.h"

#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <set>

namespace spt {

namespace {

struct ParseError {
  std::string msg;
};

// Bounds-checked little-endian reader over one mapped file.
struct Cursor {
  const uint8_t *base;
  uint64_t size, pos = 0;
  void need(uint64_t n) const {
    if (pos > size || n > size - pos) throw ParseError{"unexpected end of file"};
  }
  template <class T>
  T read() {
    need(sizeof(T));
    T v;
    memcpy(&v, base + pos, sizeof(T));
    pos += sizeof(T);
    return v;
  }
  std::string str() {  // readString (index.go:434-449)
    const uint64_t len = read<uint64_t>();
    if (len > (1u << 20)) throw ParseError{"GGUF string is too long: " + std::to_string(len)};
    need(len);
    std::string s(reinterpret_cast<const char *>(base + pos), (size_t)len);
    pos += len;
    return s;
  }
};

int meta_width(uint32_t t) {  // metadataWidth (index.go:451-463)
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
  }
}

// skipValue (index.go:465-537): returns true with *number for the unsigned
// integer scalars (the only values the index keeps as numbers).
bool skip_value(Cursor &c, uint32_t typ, int depth, uint64_t *number) {
  if (depth > 8) throw ParseError{"metadata nesting is too deep"};
  if (typ == 9) {
    const uint32_t et = c.read<uint32_t>();
    const uint64_t count = c.read<uint64_t>();
    if (count > 100000000ull) throw ParseError{"array is too large"};
    const int w = meta_width(et);
    if (w == 0 && et != 8 && et != 9) throw ParseError{"unknown metadata type " + std::to_string(et)};
    if (w != 0) {
      if (count == 0) return false;
      if (depth == 8) throw ParseError{"metadata nesting is too deep"};
      c.need(count * (uint64_t)w);
      c.pos += count * (uint64_t)w;
      return false;
    }
    for (uint64_t i = 0; i < count; ++i) {
      uint64_t unused;
      skip_value(c, et, depth + 1, &unused);
    }
    return false;
  }
  if (typ == 8) {
    c.str();
    return false;
  }
  const int w = meta_width(typ);
  if (w == 0) throw ParseError{"unknown metadata type " + std::to_string(typ)};
  c.need((uint64_t)w);
  uint64_t v = 0;
  memcpy(&v, c.base + c.pos, (size_t)w);
  c.pos += (uint64_t)w;
  if (typ == 0 || typ == 2 || typ == 4 || typ == 10) {
    *number = v;
    return true;
  }
  return false;
}

// tensorSize (index.go:539-575): elements per block and bytes per block.
bool ggml_layout(uint32_t type, uint64_t *elements, uint64_t *bytes) {
  switch (type) {
    case 0: *elements = 1; *bytes = 4; return true;    // F32
    case 1: *elements = 1; *bytes = 2; return true;    // F16
    case 2: *elements = 32; *bytes = 18; return true;  // Q4_0
    case 3: *elements = 32; *bytes = 20; return true;  // Q4_1
    case 6: *elements = 32; *bytes = 22; return true;  // Q5_0
    case 7: *elements = 32; *bytes = 24; return true;  // Q5_1
    case 8: *elements = 32; *bytes = 34; return true;  // Q8_0
    case 9: *elements = 32; *bytes = 40; return true;  // Q8_1
    case 28: *elements = 1; *bytes = 2; return true;   // BF16
    case 39: *elements = 32; *bytes = 17; return true; // MXFP4
    default: return false;
  }
}

uint64_t tensor_size(uint32_t type, const std::vector<uint64_t> &shape) {
  uint64_t per = 0, bytes = 0;
  if (!ggml_layout(type, &per, &bytes)) throw ParseError{"unsupported GGML tensor type " + std::to_string(type)};
  uint64_t n = 1;
  for (uint64_t d : shape) {
    if (d == 0 || n > UINT64_MAX / d) throw ParseError{"invalid tensor shape"};
    n *= d;
  }
  if (n % per != 0 || n / per > UINT64_MAX / bytes) throw ParseError{"invalid block size or tensor is too large"};
  return n / per * bytes;
}

// Layer number of a name "blk.N.<rest>", or -1.
int64_t layer_of(const std::string &name) {
  if (name.compare(0, 4, "blk.") != 0) return -1;
  size_t i = 4;
  while (i < name.size() && name[i] >= '0' && name[i] <= '9') ++i;
  if (i == 4 || i >= name.size() || name[i] != '.') return -1;
  if (i - 4 > 18) throw ParseError{"invalid layer number in \"" + name + "\""};
  return std::stoll(name.substr(4, i - 4));
}

void map_file(const std::string &path, GgufFile *f) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) throw ParseError{std::string("open: ") + strerror(errno)};
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    throw ParseError{std::string("stat: ") + strerror(errno)};
  }
  f->path = path;
  f->size = (uint64_t)st.st_size;
  if (f->size < 24) {
    close(fd);
    throw ParseError{"file is too small"};
  }
  void *p = mmap(nullptr, (size_t)f->size, PROT_READ, MAP_SHARED, fd, 0);
  close(fd);
  if (p == MAP_FAILED) throw ParseError{std::string("mmap: ") + strerror(errno)};
  f->base = static_cast<const uint8_t *>(p);
}

bool same_meta(const GgufModel &m, const GgufMeta &a, const GgufMeta &b) {
  if (a.type != b.type || a.end - a.start != b.end - b.start) return false;
  return memcmp(m.files[(size_t)a.file].base + a.start, m.files[(size_t)b.file].base + b.start,
                (size_t)(a.end - a.start)) == 0;
}

}  // namespace

void gguf_close(GgufModel *m) {
  for (GgufFile &f : m->files)
    if (f.base) munmap(const_cast<uint8_t *>(f.base), (size_t)f.size);
  *m = GgufModel();
}

bool gguf_open(const std::vector<std::string> &paths, GgufModel *m, std::string *err) {
  *m = GgufModel();
  if (paths.empty()) {
    *err = "no GGUF files provided";
    return false;
  }
  std::string where;
  try {
    std::set<std::string> seen_paths;
    std::set<uint64_t> split_numbers;
    int64_t declared = -1;
    uint64_t split_count = 0;
    bool has_split_count = false;
    std::map<int64_t, std::vector<size_t>> layers;
    for (const std::string &path : paths) {
      where = path + ": ";
      if (!seen_paths.insert(path).second) throw ParseError{"duplicate file"};
      const int fi = (int)m->files.size();
      m->files.emplace_back();
      map_file(path, &m->files.back());
      Cursor c{m->files.back().base, m->files.back().size};
      // header (index.go:261-291)
      if (memcmp(c.base, "GGUF", 4) != 0) throw ParseError{"not a GGUF file"};
      c.pos = 4;
      const uint32_t version = c.read<uint32_t>();
      if (version != 2 && version != 3) throw ParseError{"unsupported GGUF version " + std::to_string(version)};
      const uint64_t n_tensors = c.read<uint64_t>(), n_meta = c.read<uint64_t>();
      if (n_tensors > 10000000ull || n_meta > 1000000ull) throw ParseError{"implausible header count"};
      // metadata (index.go:293-330)
      std::map<std::string, uint64_t> numbers;
      std::map<std::string, GgufMeta> entries;
      for (uint64_t i = 0; i < n_meta; ++i) {
        const std::string key = c.str();
        if (entries.count(key)) throw ParseError{"duplicate metadata key \"" + key + "\""};
        const uint32_t typ = c.read<uint32_t>();
        GgufMeta e;
        e.type = typ;
        e.file = fi;
        e.start = c.pos;
        uint64_t num = 0;
        bool numeric = false;
        try {
          numeric = skip_value(c, typ, 0, &num);
        } catch (ParseError &pe) {
          throw ParseError{"metadata \"" + key + "\": " + pe.msg};
        }
        e.end = c.pos;
        entries[key] = e;
        if (numeric) numbers[key] = num;
      }
      // tensor directory (index.go:332-366)
      struct Info {
        std::string name;
        std::vector<uint64_t> shape;
        uint32_t type;
        uint64_t offset;
      };
      std::vector<Info> infos;
      infos.reserve((size_t)n_tensors);
      for (uint64_t i = 0; i < n_tensors; ++i) {
        Info in;
        in.name = c.str();
        const uint32_t dims = c.read<uint32_t>();
        if (dims == 0 || dims > 8) throw ParseError{"tensor \"" + in.name + "\": invalid dimension count"};
        in.shape.resize(dims);
        for (uint32_t d = 0; d < dims; ++d) in.shape[d] = c.read<uint64_t>();
        in.type = c.read<uint32_t>();
        in.offset = c.read<uint64_t>();
        infos.push_back(std::move(in));
      }
      uint64_t alignment = numbers.count("general.alignment") ? numbers["general.alignment"] : 0;
      if (alignment == 0) alignment = 32;
      if (alignment > (1u << 20) || (alignment & (alignment - 1)) != 0)
        throw ParseError{"invalid alignment " + std::to_string(alignment)};
      const uint64_t base = (c.pos + alignment - 1) & ~(alignment - 1), size = c.size;
      if (base > size) throw ParseError{"tensor data starts beyond the end of the file"};
      // model-level consistency (index.go:88-147)
      if (m->alignment == 0) m->alignment = alignment;
      else if (m->alignment != alignment) throw ParseError{"inconsistent tensor alignment"};
      for (auto &kv : entries) {
        auto it = m->meta.find(kv.first);
        if (it == m->meta.end()) {
          m->meta[kv.first] = kv.second;
          continue;
        }
        if (kv.first == "split.no") continue;
        if (!same_meta(*m, it->second, kv.second)) throw ParseError{"inconsistent metadata \"" + kv.first + "\""};
      }
      if (numbers.count("gpt_oss.block_count")) {
        const uint64_t count = numbers["gpt_oss.block_count"];
        if (count > (uint64_t)INT64_MAX) throw ParseError{"layer count is too large"};
        if (declared >= 0 && (uint64_t)declared != count) throw ParseError{"inconsistent layer count"};
        declared = (int64_t)count;
      }
      if (numbers.count("split.count")) {
        const uint64_t count = numbers["split.count"];
        if (has_split_count && split_count != count) throw ParseError{"inconsistent split count"};
        split_count = count;
        has_split_count = true;
      }
      if (numbers.count("split.no")) {
        const uint64_t no = numbers["split.no"];
        if (!split_numbers.insert(no).second) throw ParseError{"duplicate split " + std::to_string(no)};
      }
      for (const Info &in : infos) {
        uint64_t bytes = 0;
        try {
          bytes = tensor_size(in.type, in.shape);
        } catch (ParseError &pe) {
          throw ParseError{"tensor \"" + in.name + "\": " + pe.msg};
        }
        if (in.offset > size - base || bytes > size - base - in.offset)
          throw ParseError{"tensor \"" + in.name + "\": byte range extends beyond the file"};
        if (m->by_name.count(in.name)) throw ParseError{"duplicate tensor \"" + in.name + "\""};
        GgufTensor t;
        t.name = in.name;
        t.type = in.type;
        t.shape = in.shape;
        t.file = fi;
        t.start = base + in.offset;
        t.end = t.start + bytes;
        const size_t idx = m->tensors.size();
        m->by_name[t.name] = idx;
        const int64_t layer = layer_of(t.name);
        m->tensors.push_back(std::move(t));
        if (layer >= 0) layers[layer].push_back(idx);
      }
    }
    where.clear();
    // splits and layers (index.go:149-211)
    if (has_split_count && (uint64_t)paths.size() != split_count)
      throw ParseError{"incomplete model: " + std::to_string(paths.size()) + " of " + std::to_string(split_count) +
                       " splits provided"};
    if (!split_numbers.empty()) {
      if (split_numbers.size() != paths.size()) throw ParseError{"a file is missing its split number"};
      for (uint64_t n = 0; n < paths.size(); ++n)
        if (!split_numbers.count(n)) throw ParseError{"split " + std::to_string(n) + " is missing"};
    }
    if (declared < 0) declared = (int64_t)layers.size();
    if ((int64_t)layers.size() != declared)
      throw ParseError{"expected " + std::to_string(declared) + " layers, found " + std::to_string(layers.size())};
    m->layer_count = declared;
    m->layers.resize((size_t)declared);
    for (int64_t n = 0; n < declared; ++n) {
      auto it = layers.find(n);
      if (it == layers.end()) throw ParseError{"layer " + std::to_string(n) + " is missing"};
      std::vector<size_t> idx = it->second;
      std::sort(idx.begin(), idx.end(),
                [&](size_t a, size_t b) { return m->tensors[a].name < m->tensors[b].name; });
      m->layers[(size_t)n] = std::move(idx);
    }
  } catch (ParseError &pe) {
    *err = where + pe.msg;
    gguf_close(m);
    return false;
  }
  return true;
}

bool gguf_meta_int(const GgufModel &m, const std::string &key, int64_t *out) {
  auto it = m.meta.find(key);
  if (it == m.meta.end()) return false;
  const GgufMeta &e = it->second;
  const uint8_t *p = m.files[(size_t)e.file].base + e.start;
  int64_t v = 0;
  switch (e.type) {
    case 0: v = *p; break;
    case 1: v = (int8_t)*p; break;
    case 2: { uint16_t x; memcpy(&x, p, 2); v = x; break; }
    case 3: { int16_t x; memcpy(&x, p, 2); v = x; break; }
    case 4: { uint32_t x; memcpy(&x, p, 4); v = x; break; }
    case 5: { int32_t x; memcpy(&x, p, 4); v = x; break; }
    case 10: { uint64_t x; memcpy(&x, p, 8); if (x > (uint64_t)INT64_MAX) return false; v = (int64_t)x; break; }
    case 11: { int64_t x; memcpy(&x, p, 8); v = x; break; }
    case 6: case 12: {
      double d;
      if (!gguf_meta_float(m, key, &d) || d != std::floor(d) || std::fabs(d) > 9.0e18) return false;
      v = (int64_t)d;
      break;
    }
    default: return false;
  }
  *out = v;
  return true;
}

bool gguf_meta_float(const GgufModel &m, const std::string &key, double *out) {
  auto it = m.meta.find(key);
  if (it == m.meta.end()) return false;
  const GgufMeta &e = it->second;
  const uint8_t *p = m.files[(size_t)e.file].base + e.start;
  if (e.type == 6) {
    float f;
    memcpy(&f, p, 4);
    *out = f;
    return true;
  }
  if (e.type == 12) {
    memcpy(out, p, 8);
    return true;
  }
  int64_t v;
  if (e.type != 6 && e.type != 12 && e.type <= 11 && e.type != 7 && e.type != 8 && e.type != 9 &&
      gguf_meta_int(m, key, &v)) {
    *out = (double)v;
    return true;
  }
  return false;
}

}  // namespace spt
