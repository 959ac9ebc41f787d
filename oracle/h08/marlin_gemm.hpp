// marlin_gemm.hpp -- TEST INFRASTRUCTURE ONLY.  The header name that the
// reference's H08 harness (hydrogen/src/tools/bench_marlin_gemm.cpp:4)
// includes, resolved to this library's drop-in header, so that the harness
// compiles unmodified and links against libhq.so (oracle/build.py,
// build_ref_h08).
#pragma once
#include "hq_marlin_gemm.hpp"
