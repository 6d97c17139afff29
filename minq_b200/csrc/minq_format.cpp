// `.minq` reader (format.rs:1-277) for the model loader, with the same
// hardening: every length field is checked against the bytes left in the
// file before anything is allocated (format.rs:128-145), the data length
// must equal the shape-derived byte count (format.rs:212-249), and the
// legacy "MINFER01" magic is accepted (format.rs:32-35).
#include "minq_format.h"

#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace minq {

namespace {

// Bounds-checked reads from the mapped file.
struct Cursor {
  const uint8_t* base;
  uint64_t pos = 0, len = 0;
  std::string path;
  minq_status take(uint64_t n, const char* what, std::string* err) {
    uint64_t end = pos + n;
    if (end < pos) {
      *err = path + ": " + what + " length overflows";
      return MINQ_ERR_FORMAT;
    }
    if (end > len) {
      *err = path + ": " + what + " claims " + std::to_string(n) + " bytes at offset " +
             std::to_string(pos) + ", file is " + std::to_string(len) + " bytes";
      return MINQ_ERR_FORMAT;
    }
    return MINQ_OK;
  }
  // copies n bytes that take() admitted and moves past them
  void read(void* dst, uint64_t n) {
    if (n) std::memcpy(dst, base + pos, n);
    pos += n;
  }
};

}  // namespace

MinqMapping::~MinqMapping() {
  if (base) munmap(const_cast<uint8_t*>(base), len);
}

// Flat JSON object of ModelConfig (model.rs:29-45) as serde_json writes it.
minq_status parse_config_json(const std::string& s, minq_config* c, std::string* err) {
  std::map<std::string, std::string> kv;
  size_t i = 0;
  auto skip = [&] {
    while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
  };
  auto bad = [&](const char* what) {
    *err = std::string("json error: config ") + what;
    return MINQ_ERR_FORMAT;
  };
  skip();
  if (i >= s.size() || s[i] != '{') return bad("is not an object");
  ++i;
  while (true) {
    skip();
    if (i < s.size() && s[i] == '}') break;
    if (i >= s.size() || s[i] != '"') return bad("expected a key");
    size_t e = s.find('"', i + 1);
    if (e == std::string::npos) return bad("has an unterminated key");
    std::string key = s.substr(i + 1, e - i - 1);
    i = e + 1;
    skip();
    if (i >= s.size() || s[i] != ':') return bad("expected ':'");
    ++i;
    skip();
    std::string val;
    if (i < s.size() && s[i] == '"') {
      size_t e2 = s.find('"', i + 1);
      if (e2 == std::string::npos) return bad("has an unterminated string");
      val = s.substr(i + 1, e2 - i - 1);
      i = e2 + 1;
    } else {
      size_t st = i;
      while (i < s.size() && s[i] != ',' && s[i] != '}') ++i;
      val = s.substr(st, i - st);
      while (!val.empty() && std::isspace(static_cast<unsigned char>(val.back()))) val.pop_back();
    }
    kv[key] = val;
    skip();
    if (i < s.size() && s[i] == ',') {
      ++i;
      continue;
    }
    if (i < s.size() && s[i] == '}') break;
    return bad("expected ',' or '}'");
  }
  static const char* need[] = {"hidden_size", "intermediate_size", "n_layers", "n_heads",
                               "n_kv_heads", "head_dim", "vocab_size", "max_seq_len",
                               "rope_theta", "rms_norm_eps", "has_qkv_bias", "dtype"};
  for (const char* k : need) {
    if (!kv.count(k)) {
      *err = std::string("json error: missing field `") + k + "`";
      return MINQ_ERR_FORMAT;
    }
  }
  auto u = [&](const char* k) { return (uint64_t)std::strtoull(kv[k].c_str(), nullptr, 10); };
  c->hidden_size = u("hidden_size");
  c->intermediate_size = u("intermediate_size");
  c->n_layers = u("n_layers");
  c->n_heads = u("n_heads");
  c->n_kv_heads = u("n_kv_heads");
  c->head_dim = u("head_dim");
  c->vocab_size = u("vocab_size");
  c->max_seq_len = u("max_seq_len");
  c->rope_theta = (float)std::strtod(kv["rope_theta"].c_str(), nullptr);
  c->rms_norm_eps = (float)std::strtod(kv["rms_norm_eps"].c_str(), nullptr);
  c->has_qkv_bias = kv["has_qkv_bias"] == "true";
  const std::string& d = kv["dtype"];
  c->dtype = d == "q8_0" ? MINQ_Q8_0 : (d == "q4_0" ? MINQ_Q4_0 : MINQ_F32);
  return MINQ_OK;
}

minq_status index_minq_file(const std::string& path, minq_config* cfg,
                            std::vector<MinqRecord>* records, MinqMapping* map,
                            std::string* err) {
  const int fd = open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    *err = "io error: cannot open " + path;
    return MINQ_ERR_IO;
  }
  struct stat sb;
  if (fstat(fd, &sb) != 0) {
    close(fd);
    *err = "io error: cannot stat " + path;
    return MINQ_ERR_IO;
  }
  const uint64_t flen = (uint64_t)sb.st_size;
  if (flen > 0) {
    void* a = mmap(nullptr, flen, PROT_READ, MAP_PRIVATE, fd, 0);
    if (a == MAP_FAILED) {
      close(fd);
      *err = "io error: cannot map " + path;
      return MINQ_ERR_IO;
    }
    madvise(a, flen, MADV_SEQUENTIAL);
    map->base = static_cast<const uint8_t*>(a);
    map->len = flen;
  }
  close(fd);  // the mapping keeps the file
  Cursor r;
  r.base = map->base;
  r.len = flen;
  r.path = path;
  minq_status st;
  if ((st = r.take(8, "magic", err))) return st;
  char magic[8];
  r.read(magic, 8);
  if (std::memcmp(magic, "MINQ0001", 8) != 0 && std::memcmp(magic, "MINFER01", 8) != 0) {
    *err = path + ": not a .minq/.minfer file (bad magic)";
    return MINQ_ERR_FORMAT;
  }
  if ((st = r.take(4, "config length", err))) return st;
  uint32_t cfg_len;
  r.read(&cfg_len, 4);
  if ((st = r.take(cfg_len, "config json", err))) return st;
  std::string js(cfg_len, '\0');
  r.read(&js[0], cfg_len);
  if ((st = parse_config_json(js, cfg, err))) return st;
  while (r.pos < r.len) {  // clean EOF between records (format.rs:173-177)
    if ((st = r.take(4, "tensor name length", err))) return st;
    uint32_t name_len;
    r.read(&name_len, 4);
    if ((st = r.take(name_len, "tensor name", err))) return st;
    MinqRecord rec;
    rec.name.assign(name_len, '\0');
    r.read(&rec.name[0], name_len);
    if ((st = r.take(2, "tensor tag/ndim", err))) return st;
    uint8_t tag, ndim;
    r.read(&tag, 1);
    r.read(&ndim, 1);
    if ((st = r.take(8ull * ndim, "tensor shape", err))) return st;
    rec.shape.resize(ndim);
    r.read(rec.shape.data(), 8ull * ndim);
    uint64_t numel = 1;
    for (uint64_t d : rec.shape) {
      if (d != 0 && numel > UINT64_MAX / d) {
        *err = "tensor `" + rec.name + "`: shape overflows usize";
        return MINQ_ERR_FORMAT;
      }
      numel *= d;
    }
    if ((st = r.take(8, "tensor data length", err))) return st;
    uint64_t data_len;
    r.read(&data_len, 8);
    uint64_t expected = 0;
    if (tag == MINQ_F32) {
      if (numel > UINT64_MAX / 4) {
        *err = "tensor `" + rec.name + "`: byte count overflows";
        return MINQ_ERR_FORMAT;
      }
      expected = numel * 4;
    } else if (tag == MINQ_Q8_0 || tag == MINQ_Q4_0) {
      if (ndim != 2) {
        *err = "quantized tensor `" + rec.name + "` must be 2-D";
        return MINQ_ERR_FORMAT;
      }
      uint64_t rows = rec.shape[0], cols = rec.shape[1];
      if (cols % 32 != 0) {
        *err = "quantized tensor `" + rec.name + "`: cols " + std::to_string(cols) +
               " not block-aligned";
        return MINQ_ERR_FORMAT;
      }
      uint64_t nb = cols / 32, bb = tag == MINQ_Q8_0 ? 36 : 20;
      if ((nb != 0 && rows > UINT64_MAX / nb) || rows * nb > UINT64_MAX / bb) {
        *err = "tensor `" + rec.name + "`: byte count overflows";
        return MINQ_ERR_FORMAT;
      }
      expected = rows * nb * bb;
    } else {
      *err = "tensor `" + rec.name + "`: unknown storage tag " + std::to_string(tag);
      return MINQ_ERR_FORMAT;
    }
    if (data_len != expected) {
      *err = "tensor `" + rec.name + "`: data length " + std::to_string(data_len) +
             " != shape-derived " + std::to_string(expected);
      return MINQ_ERR_FORMAT;
    }
    if ((st = r.take(data_len, "tensor data", err))) return st;
    rec.tag = tag;
    rec.offset = r.pos;
    rec.nbytes = data_len;
    r.pos += data_len;
    records->push_back(std::move(rec));
  }
  return MINQ_OK;
}

}  // namespace minq
