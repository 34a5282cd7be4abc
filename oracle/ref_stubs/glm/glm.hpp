// Minimal vector types standing in for glm when the reference world generator
// is compiled as a test oracle. Only construction, member access, +, - and ==
// are provided: the generation/lighting path does no glm arithmetic beyond
// moving coordinates around (reference: src/world/WorldGenerator.cu,
// src/world/WorldGenerator.h, include/blocklab/utility/Math.h).
//
// Test infrastructure only; never linked into the product library.
#pragma once

#include <cstdint>

namespace glm {

template <typename T>
struct tvec2 {
    T x {}, y {};
    constexpr tvec2() = default;
    constexpr tvec2(T a, T b) : x(a), y(b) {}
    constexpr T operator[](int i) const { return i == 0 ? x : y; }
    friend constexpr bool operator==(const tvec2& a, const tvec2& b) { return a.x == b.x && a.y == b.y; }
};

template <typename T>
struct tvec3 {
    T x {}, y {}, z {};
    constexpr tvec3() = default;
    constexpr explicit tvec3(T s) : x(s), y(s), z(s) {}
    constexpr tvec3(T a, T b, T c) : x(a), y(b), z(c) {}
    template <typename U>
    constexpr explicit tvec3(const tvec3<U>& o) : x(static_cast<T>(o.x)), y(static_cast<T>(o.y)), z(static_cast<T>(o.z)) {}
    friend constexpr tvec3 operator+(tvec3 a, const tvec3& b) { return { a.x + b.x, a.y + b.y, a.z + b.z }; }
    friend constexpr tvec3 operator-(tvec3 a, const tvec3& b) { return { a.x - b.x, a.y - b.y, a.z - b.z }; }
    friend constexpr bool operator==(const tvec3& a, const tvec3& b) { return a.x == b.x && a.y == b.y && a.z == b.z; }
};

template <typename T>
struct tvec4 {
    T x {}, y {}, z {}, w {};
    constexpr tvec4() = default;
    constexpr tvec4(T a, T b, T c, T d) : x(a), y(b), z(c), w(d) {}
};

using vec2 = tvec2<float>;
using vec3 = tvec3<float>;
using vec4 = tvec4<float>;
using ivec2 = tvec2<std::int32_t>;
using ivec3 = tvec3<std::int32_t>;
using ivec4 = tvec4<std::int32_t>;
using uvec3 = tvec3<std::uint32_t>;

} // namespace glm
