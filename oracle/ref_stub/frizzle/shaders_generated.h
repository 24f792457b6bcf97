// Stands in for the header the reference's build generates from its WGSL
// (cmake/embed_shaders_script.cmake), so that capture.cpp compiles here for
// the test-only shim: capture::layout() reads no shader, and the launches
// that name these two kernels are never built by the shim.
#pragma once

#include <string_view>

namespace frizzle::shaders {
inline constexpr std::string_view capture{};
inline constexpr std::string_view weights{};
}  // namespace frizzle::shaders
