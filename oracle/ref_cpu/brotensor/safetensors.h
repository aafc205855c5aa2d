// CPU stand-in (checker only): the reference's headers name this type in
// load_from() declarations, which the checker never calls.
#pragma once

namespace brotensor {
namespace safetensors {
class File;
}
}  // namespace brotensor
