// spt_gguf.h -- GGUF model index (host only): headers, metadata and tensor
// directories of one model, split files in any order, mapped read-only.
// The rules follow ggufindex.Open (ggufindex/index.go:55-575):
//   * magic "GGUF", version 2 or 3, at most 10,000,000 tensors and
//     1,000,000 metadata entries per file; no duplicate keys;
//   * metadata values of every GGUF type, arrays nested at most 8 deep;
//   * alignment = general.alignment (default 32), a power of two <= 1 MiB,
//     the same in every file; tensor data starts at the aligned end of the
//     tensor directory;
//   * tensor sizes from the GGML type table (F32, F16, Q4_0, Q4_1, Q5_0,
//     Q5_1, Q8_0, Q8_1, BF16, MXFP4), every byte range inside its file;
//   * no duplicate tensor names across files; split.count / split.no
//     consistent and complete; metadata shared by the files identical;
//   * tensors named blk.N.* belong to layer N; the layer count is
//     gpt_oss.block_count when present, else the number of layers found, and
//     every layer below it must exist.
#pragma once
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace spt {

struct GgufTensor {
  std::string name;
  uint32_t type = 0;
  std::vector<uint64_t> shape;
  int file = 0;                  // index into GgufModel::files
  uint64_t start = 0, end = 0;   // absolute byte range in that file
};

struct GgufMeta {
  uint32_t type = 0;
  int file = 0;
  uint64_t start = 0, end = 0;  // encoded value (after the type tag)
};

struct GgufFile {
  std::string path;
  const uint8_t *base = nullptr;  // read-only mapping of the whole file
  uint64_t size = 0;
};

struct GgufModel {
  std::vector<GgufFile> files;
  std::vector<GgufTensor> tensors;
  std::map<std::string, size_t> by_name;            // tensor index
  std::vector<std::vector<size_t>> layers;          // tensor indices per layer, sorted by name
  std::map<std::string, GgufMeta> meta;
  uint64_t alignment = 0;
  int64_t layer_count = 0;
};

// Returns false and sets *err on a malformed or inconsistent model (the
// mappings made so far are released).
bool gguf_open(const std::vector<std::string> &paths, GgufModel *m, std::string *err);
void gguf_close(GgufModel *m);
// Integer (any integer type) / float (F32 or F64) metadata value.
bool gguf_meta_int(const GgufModel &m, const std::string &key, int64_t *out);
bool gguf_meta_float(const GgufModel &m, const std::string &key, double *out);

}  // namespace spt
