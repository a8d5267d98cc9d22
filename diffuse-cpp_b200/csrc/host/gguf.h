// GGUF v2/v3 reader (mmap) and streaming writer for the host library.
// Format as written by gguf-py's GGUFWriter, which the reference's converters use
// (tools/convert-llada.py:185-202, tools/convert-dream.py:180-195).
#pragma once
#include <cstdint>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

namespace dfh {

enum GgmlType : int32_t { GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_Q4_K = 12, GT_Q6_K = 14, GT_BF16 = 30 };
int64_t ggml_block_size(int32_t t);
int64_t ggml_type_size(int32_t t);
int64_t ggml_row_size(int32_t t, int64_t n);
const char *ggml_type_name(int32_t t);

struct GgufValue {
    int32_t type = -1;  // GGUF value type
    uint64_t u = 0;
    double f = 0;
    std::string s;
};

struct GgufTensor {
    std::string name;
    int32_t type = 0;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;
    const uint8_t *data = nullptr;
    size_t nbytes = 0;
};

class GgufReader {
  public:
    ~GgufReader();
    bool open(const std::string &path, std::string *err);
    const GgufValue *find(const std::string &key) const;
    const GgufTensor *tensor(const std::string &name) const;
    const std::vector<GgufTensor> &tensors() const { return tensors_; }
    const std::map<std::string, GgufValue> &kv() const { return kv_; }

  private:
    void *map_ = nullptr;
    size_t size_ = 0;
    std::map<std::string, GgufValue> kv_;
    std::vector<GgufTensor> tensors_;
    std::map<std::string, size_t> index_;
};

// Writes a GGUF v3 file: all metadata and tensor infos first, then tensor data
// appended in declaration order (so multi-GB models stream through memory).
class GgufWriter {
  public:
    void add_u32(const std::string &k, uint32_t v);
    void add_f32(const std::string &k, float v);
    void add_str(const std::string &k, const std::string &v);
    void add_tensor_info(const std::string &name, int32_t type, int n_dims, const int64_t *ne);
    bool begin(const std::string &path, std::string *err);                  // header + kv + infos
    bool write_tensor_data(const void *data, size_t nbytes, std::string *err);  // next tensor, in order
    bool finish(std::string *err);

  private:
    struct KV { std::string key; int32_t type; uint32_t u; float f; std::string s; };
    struct TI { std::string name; int32_t type; int n_dims; int64_t ne[4]; uint64_t offset; size_t nbytes; };
    std::vector<KV> kv_;
    std::vector<TI> ti_;
    FILE *f_ = nullptr;
    size_t next_ = 0;
    uint64_t data_bytes_ = 0;
};

}  // namespace dfh
