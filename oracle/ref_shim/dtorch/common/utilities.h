// Shim (oracle build): the helpers the reference thread-group sources use from dtorch/common/utilities.h.
#pragma once
#include <type_traits>
#include <utility>

#include "dtorch/common/debug.h"

#define DTORCH_FORCEINLINE inline
#define DTORCH_API_FORCEINLINE inline
#define DTORCH_DISABLE_COPY_AND_MOVE(T) \
    T(const T&) = delete;               \
    T& operator=(const T&) = delete;    \
    T(T&&) = delete;                    \
    T& operator=(T&&) = delete
#define DTORCH_API_DISABLE_COPY_AND_MOVE(T) DTORCH_DISABLE_COPY_AND_MOVE(T)

namespace dtorch {
template <typename... Ts>
inline void IgnoreUnused(Ts&&...) {}

template <typename E>
constexpr auto EnumAsInteger(E e) { return static_cast<std::underlying_type_t<E>>(e); }
}  // namespace dtorch
