// CPU stand-in (checker only).
#pragma once

namespace brotensor {
inline void init() {}
}  // namespace brotensor
