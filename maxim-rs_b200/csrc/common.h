// Shared error plumbing for the host library.
//
// The reference's error type is a single string (`Error(String)`, src/lib.rs:29-56)
// propagated to `main`, which prints `maxim: {e}` and exits 1. Inside this
// library the same thing is a C++ exception carrying the message and an ABI
// status code; every extern "C" entry point catches it, stores the message in
// a thread-local slot (read back with mx_last_error) and returns the code.
#pragma once

#include <stdexcept>
#include <string>

#include "maxim_b200.h"

namespace mx {

struct Error : std::runtime_error {
  int code;
  explicit Error(const std::string& msg, int c = MX_E_INVALID) : std::runtime_error(msg), code(c) {}
};

void set_last_error(const std::string& msg);

// Run `f` and translate any exception into a status code.
template <class F>
int guard(F&& f) {
  try {
    f();
    return MX_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return MX_E_OOM;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return MX_E_INVALID;
  }
}

// printf-style string building for messages.
std::string fmt(const char* f, ...) __attribute__((format(printf, 1, 2)));

}  // namespace mx
