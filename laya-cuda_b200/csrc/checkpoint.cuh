// Checkpoint loading: the safetensors header parser and the device-side conversion kernel used by
// laya_load_checkpoint (laya_b200.cu).
//
// A safetensors file is an 8-byte little-endian header length N, N bytes of JSON
//   {"<name>": {"dtype": "F32"|"F16"|"BF16"|..., "shape": [..], "data_offsets": [begin, end]},
//    ..., "__metadata__": {"<key>": "<value>", ...}}
// and the tensor bytes, each tensor at [8 + N + begin, 8 + N + end), row-major, little-endian.
// The reference reads it through the safetensors library and uploads tensor by tensor
// (laya_cuda/runtime.py:147-158); here the file is mapped once, raw chunks are staged in pinned
// memory and uploaded asynchronously, and the conversion to the stored type (16-bit GEMM
// operands, fp32 for the rest) and the GeGLU row interleave run on the device.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace laya {

enum class StDtype : int { F32 = 0, F16 = 1, BF16 = 2 };

struct StEntry {
  StDtype dtype = StDtype::F32;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte offsets into the data section
};

// Minimal JSON reader for a safetensors header: objects, arrays, strings (with escapes),
// integers, true / false / null.  Throws std::runtime_error on malformed input.
class StHeaderParser {
 public:
  StHeaderParser(const char* text, size_t size) : p_(text), end_(text + size) {}

  std::map<std::string, StEntry> parse() {
    std::map<std::string, StEntry> out;
    ws();
    expect('{');
    ws();
    if (peek() == '}') { ++p_; return out; }
    for (;;) {
      ws();
      const std::string name = str();
      ws();
      expect(':');
      ws();
      if (name == "__metadata__") skip_value();
      else out[name] = entry(name);
      ws();
      if (peek() == ',') { ++p_; continue; }
      expect('}');
      break;
    }
    return out;
  }

 private:
  const char* p_;
  const char* end_;

  [[noreturn]] void bad(const char* what) { throw std::runtime_error(std::string("safetensors header: ") + what); }
  char peek() { return p_ < end_ ? *p_ : '\0'; }
  void expect(char c) {
    if (peek() != c) bad("unexpected character");
    ++p_;
  }
  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
  }
  std::string str() {
    expect('"');
    std::string s;
    while (p_ < end_ && *p_ != '"') {
      char c = *p_++;
      if (c != '\\') { s.push_back(c); continue; }
      if (p_ >= end_) bad("truncated escape");
      const char e = *p_++;
      switch (e) {
        case '"': case '\\': case '/': s.push_back(e); break;
        case 'b': s.push_back('\b'); break;
        case 'f': s.push_back('\f'); break;
        case 'n': s.push_back('\n'); break;
        case 'r': s.push_back('\r'); break;
        case 't': s.push_back('\t'); break;
        case 'u': {
          if (end_ - p_ < 4) bad("truncated \\u escape");
          unsigned v = 0;
          for (int i = 0; i < 4; ++i) {
            const char h = *p_++;
            v = v * 16 + (h >= '0' && h <= '9' ? h - '0' : h >= 'a' && h <= 'f' ? h - 'a' + 10
                                                        : h >= 'A' && h <= 'F' ? h - 'A' + 10 : 99);
            if (v > 0xFFFF) bad("bad \\u escape");
          }
          // UTF-8 of the code unit (names in this format are ASCII in practice).
          if (v < 0x80) s.push_back((char)v);
          else if (v < 0x800) { s.push_back((char)(0xC0 | (v >> 6))); s.push_back((char)(0x80 | (v & 0x3F))); }
          else {
            s.push_back((char)(0xE0 | (v >> 12)));
            s.push_back((char)(0x80 | ((v >> 6) & 0x3F)));
            s.push_back((char)(0x80 | (v & 0x3F)));
          }
          break;
        }
        default: bad("unknown escape");
      }
    }
    expect('"');
    return s;
  }
  int64_t integer() {
    bool neg = false;
    if (peek() == '-') { neg = true; ++p_; }
    if (!(peek() >= '0' && peek() <= '9')) bad("expected an integer");
    int64_t v = 0;
    while (peek() >= '0' && peek() <= '9') {
      if (v > (INT64_MAX - 9) / 10) bad("integer overflow");
      v = v * 10 + (*p_++ - '0');
    }
    if (peek() == '.' || peek() == 'e' || peek() == 'E') bad("expected an integer");
    return neg ? -v : v;
  }
  std::vector<int64_t> int_array() {
    std::vector<int64_t> v;
    expect('[');
    ws();
    if (peek() == ']') { ++p_; return v; }
    for (;;) {
      ws();
      v.push_back(integer());
      ws();
      if (peek() == ',') { ++p_; continue; }
      expect(']');
      return v;
    }
  }
  void skip_value() {
    ws();
    const char c = peek();
    if (c == '"') { str(); return; }
    if (c == '{' || c == '[') {
      const char close = c == '{' ? '}' : ']';
      ++p_;
      ws();
      if (peek() == close) { ++p_; return; }
      for (;;) {
        ws();
        if (c == '{') { str(); ws(); expect(':'); }
        skip_value();
        ws();
        if (peek() == ',') { ++p_; continue; }
        expect(close);
        return;
      }
    }
    if (c == '-' || (c >= '0' && c <= '9')) {
      while (p_ < end_ && strchr("+-0123456789.eE", *p_)) ++p_;
      return;
    }
    for (const char* word : {"true", "false", "null"}) {
      const size_t n = strlen(word);
      if ((size_t)(end_ - p_) >= n && !strncmp(p_, word, n)) { p_ += n; return; }
    }
    bad("unexpected value");
  }
  StEntry entry(const std::string& name) {
    StEntry e;
    bool has_dtype = false, has_shape = false, has_offsets = false;
    expect('{');
    for (;;) {
      ws();
      const std::string key = str();
      ws();
      expect(':');
      ws();
      if (key == "dtype") {
        const std::string d = str();
        if (d == "F32") e.dtype = StDtype::F32;
        else if (d == "F16") e.dtype = StDtype::F16;
        else if (d == "BF16") e.dtype = StDtype::BF16;
        else throw std::runtime_error("unsupported dtype " + d + " of tensor " + name);
        has_dtype = true;
      } else if (key == "shape") {
        e.shape = int_array();
        for (int64_t v : e.shape)
          if (v < 0) bad("negative dimension");
        has_shape = true;
      } else if (key == "data_offsets") {
        const std::vector<int64_t> o = int_array();
        if (o.size() != 2 || o[0] < 0 || o[1] < o[0]) bad("bad data_offsets");
        e.begin = (uint64_t)o[0];
        e.end = (uint64_t)o[1];
        has_offsets = true;
      } else {
        skip_value();
      }
      ws();
      if (peek() == ',') { ++p_; continue; }
      expect('}');
      break;
    }
    if (!has_dtype || !has_shape || !has_offsets) throw std::runtime_error("incomplete header entry of " + name);
    return e;
  }
};

inline int st_dtype_bytes(StDtype d) { return d == StDtype::F32 ? 4 : 2; }

// Stored element types of the conversion kernel.
enum : int { kStoreF32 = 0, kStoreF16 = 1, kStoreBF16 = 2 };

__device__ __forceinline__ float st_load(const void* src, int dtype, int64_t i) {
  if (dtype == (int)StDtype::F32) return static_cast<const float*>(src)[i];
  if (dtype == (int)StDtype::F16) return __half2float(static_cast<const __half*>(src)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
}

// dst rows (row0 .. row0 + rows) of a [*][cols] tensor = converted src (the chunk's rows,
// contiguous).  interleave_f > 0: GeGLU rows -- source row r of a [2F][cols] tensor goes to row
// (r mod F) / 64 * 128 + (r >= F) * 64 + r mod 64, so each 128-row block holds 64 gate rows and
// their 64 up rows.  Conversions round to nearest even; fp32 -> fp32 copies.
__global__ void __launch_bounds__(256) convert_rows_kernel(const void* src, int src_dtype, void* dst, int dst_type,
                                                           int64_t row0, int64_t rows, int64_t cols,
                                                           int64_t interleave_f) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = row0 + i / cols, c = i - (i / cols) * cols;
    int64_t dr = r;
    if (interleave_f > 0) {
      const int64_t half = r >= interleave_f ? 1 : 0, rr = r - half * interleave_f;
      dr = (rr / 64) * 128 + half * 64 + rr % 64;
    }
    const float v = st_load(src, src_dtype, i);
    const int64_t o = dr * cols + c;
    if (dst_type == kStoreF32) static_cast<float*>(dst)[o] = v;
    else if (dst_type == kStoreF16) static_cast<__half*>(dst)[o] = __float2half_rn(v);
    else static_cast<__nv_bfloat16*>(dst)[o] = __float2bfloat16_rn(v);
  }
}

}  // namespace laya
