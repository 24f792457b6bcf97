// Stand-in for the reference's src/core/kernels/program.h when compiling the
// CudaProgram adapter of INTEGRATION.md: that header includes WebGPU (Dawn),
// which is not present.  It declares only what the adapter uses, with the
// reference's own declarations (program.h:264-299): the error enum and the
// step callback's signature.  Test infrastructure.
#pragma once

#include <cstddef>
#include <cstdint>
#include <span>
#include <string_view>

#include "core/kernels/interface.h"

namespace frizzle::kernels {

enum class ProgramError : std::uint8_t { Ok, Build, Step, DeviceLost, Cancelled };

using StepCallback = void (*)(ProgramError error, std::string_view message, std::span<const std::byte> readback,
                              void* userdata);

}  // namespace frizzle::kernels
