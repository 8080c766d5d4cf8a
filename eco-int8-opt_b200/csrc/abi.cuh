// Host-side helpers shared by the C-ABI entry points: thread-local error
// message, argument checks, launch checks.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#include "../../include/ecoint8_b200.h"

int eco_fail(int code, const char* fmt, ...);
int eco_launch_check(const char* what);
int eco_num_sms();

#define ECO_REQUIRE(cond, code, ...)         \
  do {                                       \
    if (!(cond)) return eco_fail(code, __VA_ARGS__); \
  } while (0)

static inline bool eco_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
static inline cudaStream_t eco_stream(eco_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Validates an SR spec for a requant with the given shift; replay needs a tensor.
int eco_check_sr(const eco_sr_t& sr, int shift, const char* who);
