// fd_trace.h - host-side trace ranges around the library's launches.
//
// Each call that launches work opens one NVTX push/pop range in the domain
// "flashdecode", named for the work ("decode", "decode_e4m3", "append",
// "append_e4m3", "exchange", "combine_lse"), so a timeline tool shows where
// a step spends its time and a kernel profiler can select this library's
// launches by range, e.g.
//   ncu --nvtx --nvtx-include "flashdecode@decode/" ...
// The reference times its kernels only from the host (torch.profiler and
// wall clock in its evaluator, evaluate_flashattn_submission.py:168-197).
//
// NVTX v3 is header-only.  With no tool attached, the first push looks for
// an injection library once and every later push/pop is a test of a null
// function pointer; nothing here allocates device memory.
#pragma once

#include <nvtx3/nvToolsExt.h>

namespace fd {

inline nvtxDomainHandle_t trace_domain() {
  static const nvtxDomainHandle_t domain = nvtxDomainCreateA("flashdecode");
  return domain;
}

// Scoped range: pushed on construction, popped when the call returns
// (whichever return it takes).  `name` must outlive the range.
class TraceRange {
 public:
  explicit TraceRange(const char* name) {
    nvtxEventAttributes_t a = {};
    a.version = NVTX_VERSION;
    a.size = NVTX_EVENT_ATTRIB_STRUCT_SIZE;
    a.messageType = NVTX_MESSAGE_TYPE_ASCII;
    a.message.ascii = name;
    nvtxDomainRangePushEx(trace_domain(), &a);
  }
  ~TraceRange() { nvtxDomainRangePop(trace_domain()); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

}  // namespace fd
