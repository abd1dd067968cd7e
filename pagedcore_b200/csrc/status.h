// Thread-local error message of the C ABI (pkv_last_error) and the helper
// that records a failure and returns its status code.
#pragma once

#include <string>

namespace pkv {

std::string &error_message();

inline void clear_error() { error_message().clear(); }

inline int fail(int code, const std::string &message) {
    error_message() = message;
    return code;
}

}  // namespace pkv
