// host_util.h - host-side helpers shared by the library's translation units.
#pragma once

#include <string>

namespace lstk {

// Records `msg` as this thread's last error and returns `code` (a negative LSTK_ERR_* value).
int set_error(int code, const std::string &msg);
// Clears this thread's last error; returns 0 (LSTK_OK).
int clear_error();

}  // namespace lstk
