// Shared by the host-side translation units of libgpeed_moe.so: records the
// message gpeed_last_error() returns on this thread and passes `code` through.
#pragma once
#include <string>

namespace gp {
int set_error(int code, const std::string& msg);
}  // namespace gp
