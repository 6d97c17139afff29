// Host-side `.minq` reader used by minq_model_load (format.rs:149-277).
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/minq_cuda.h"

namespace minq {

struct MinqRecord {
  std::string name;
  int tag = 0;
  std::vector<uint64_t> shape;
  std::vector<uint8_t> data;
};

minq_status parse_config_json(const std::string& json, minq_config* cfg, std::string* err);
minq_status read_minq_file(const std::string& path, minq_config* cfg,
                           std::vector<MinqRecord>* records, std::string* err);

}  // namespace minq
