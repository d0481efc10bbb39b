// Status codes returned by every zcutlass entry point.
//
// Mirrors the reference enum (include/zcutlass/status.hpp:5-12 in
// supercatking/zcutlass): same names, same order, so integer values match and
// callers compiled against the reference keep working.
#pragma once

namespace zcutlass {

enum class Status {
  Success,          // 0: work enqueued (or nothing to do for an empty problem)
  InvalidArgument,  // 1: negative sizes, null required pointers, ld too small
  NotSupported,     // 2: dtype / layout / shape outside what any kernel handles
  RuntimeError,     // 3: launch failed, or a kernel reported a device-side timeout
};

const char* status_to_string(Status status);

}  // namespace zcutlass
