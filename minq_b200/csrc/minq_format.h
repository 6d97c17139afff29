// Host-side `.minq` reader used by minq_model_load (format.rs:149-277): the
// file is mapped read-only and indexed in place, so tensor bytes are read
// once, from the mapping, by the uploader.
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/minq_cuda.h"

namespace minq {

// One tensor record: its header fields and where its data lies in the file.
struct MinqRecord {
  std::string name;
  int tag = 0;
  std::vector<uint64_t> shape;
  uint64_t offset = 0;  // of the data, from the start of the file
  uint64_t nbytes = 0;
};

// A read-only private mapping of a whole file (unmapped on destruction).
struct MinqMapping {
  const uint8_t* base = nullptr;
  uint64_t len = 0;
  MinqMapping() = default;
  MinqMapping(const MinqMapping&) = delete;
  MinqMapping& operator=(const MinqMapping&) = delete;
  ~MinqMapping();
};

minq_status parse_config_json(const std::string& json, minq_config* cfg, std::string* err);
// Maps `path` and indexes its records with the reader's checks (every length
// against the bytes left, data length == shape-derived bytes, known tags).
minq_status index_minq_file(const std::string& path, minq_config* cfg,
                            std::vector<MinqRecord>* records, MinqMapping* map,
                            std::string* err);

}  // namespace minq
