// api_export.cuh — include the public headers with default visibility: the library is
// built with -fvisibility=hidden so that only the C API is exported.
#pragma once
#pragma GCC visibility push(default)
#include "../../include/acfun/acfun.h"
#include "../../include/acfun/acfun_internal.h"
#pragma GCC visibility pop
