// CPU stand-in (checker only): every op the reference's decoder sources call is
// declared in brotensor/cpu_ops.h.
#pragma once
#include <brotensor/cpu_ops.h>
