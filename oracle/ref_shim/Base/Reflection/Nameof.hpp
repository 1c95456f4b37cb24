// Include-path shim used only when compiling the reference CPU path for the
// oracle.  It pulls in the reference's own Base/Reflection/Nameof.hpp
// unchanged, but with static_assert turned into a no-op for the duration of
// that one header: four of its compile-time self-checks assume the MSVC/Clang
// spelling of std::source_location::function_name() and fail under GCC, and
// nothing on the Tensor CPU path uses the names they check.
#pragma once
#include <array>
#include <bit>
#include <limits>
#include <optional>
#include <source_location>
#include <string>
#include <string_view>
#include <type_traits>
#include <utility>
#include "Base/String/Ascii.hpp"
#include "Base/String/Naming.hpp"
#include "Base/String/Text.hpp"
#define static_assert(...) static_assert(true, "")
#include BEE_REF_NAMEOF_HEADER
#undef static_assert
