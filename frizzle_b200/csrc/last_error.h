// The calling thread's last error message, read by fz_last_error().
#pragma once

namespace fz {
void set_last_error(const char* message);
}  // namespace fz
