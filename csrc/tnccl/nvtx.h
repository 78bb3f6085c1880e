// nvtx.h - optional NVTX ranges around the host entry points (TNCCL_NVTX=1),
// so a timeline tool shows each init, enqueue and destroy with its algorithm
// and size. Off by default: then a range costs one predictable branch and
// nothing is formatted.
#pragma once

#include <stdio.h>

#include <nvtx3/nvToolsExt.h>

#include "common.h"

namespace tnccl {

inline bool nvtxEnabled() {
  static const bool on = envInt("TNCCL_NVTX", 0) != 0;
  return on;
}

class NvtxRange {
 public:
  NvtxRange(const char* fmt, ...) __attribute__((format(printf, 2, 3))) {
    if (!nvtxEnabled()) return;
    char buf[160];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    nvtxRangePushA(buf);
    active_ = true;
  }
  ~NvtxRange() {
    if (active_) nvtxRangePop();
  }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;

 private:
  bool active_ = false;
};

}  // namespace tnccl
