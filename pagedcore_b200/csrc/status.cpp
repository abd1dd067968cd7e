#include "status.h"

#include "pagedkv.h"

namespace pkv {

std::string &error_message() {
    thread_local std::string message;
    return message;
}

}  // namespace pkv

extern "C" const char *pkv_last_error(void) { return pkv::error_message().c_str(); }
