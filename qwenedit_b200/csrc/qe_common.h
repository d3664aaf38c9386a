// Shared host-side helpers for libqeb200: thread-local error text and status returns.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <string>

#include "qeb200.h"

namespace qe {

// Thread-local message of the last failing call (qe_last_error).
std::string &last_error();

// Record a formatted message and return `status`.
int fail(int status, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

inline int ok() {
  last_error().clear();
  return QE_OK;
}

}  // namespace qe

#define QE_CHECK_ARG(cond, ...)                         \
  do {                                                  \
    if (!(cond)) return ::qe::fail(QE_ERR_INVALID, __VA_ARGS__); \
  } while (0)
