// Minimal vector types standing in for glm when the reference world generator
// and sky functions are compiled as a test oracle: construction, member
// access, +, -, scalar *, == and the three functions below. The generation /
// lighting path does no glm arithmetic beyond moving coordinates around
// (reference: src/world/WorldGenerator.cu, src/world/WorldGenerator.h,
// include/blocklab/utility/Math.h, src/world/Lighting.cpp).
//
// Test infrastructure only; never linked into the product library.
#pragma once

#include <cmath>
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
    friend constexpr tvec3 operator-(const tvec3& a) { return { -a.x, -a.y, -a.z }; }
    friend constexpr tvec3 operator*(const tvec3& a, T s) { return { a.x * s, a.y * s, a.z * s }; }
    friend constexpr bool operator==(const tvec3& a, const tvec3& b) { return a.x == b.x && a.y == b.y && a.z == b.z; }
};

template <typename T>
struct tvec4 {
    T x {}, y {}, z {}, w {};
    constexpr tvec4() = default;
    constexpr tvec4(T a, T b, T c, T d) : x(a), y(b), z(c), w(d) {}
};

// The few functions the reference's sky colour and light direction use
// (src/world/Lighting.cpp:53-112), written to glm's published formulas:
// mix(x, y, a) = x * (1 - a) + y * a; smoothstep clamps (x - e0) / (e1 - e0)
// to [0, 1] and returns t * t * (3 - 2 * t); normalize(v) = v * (1 / sqrt(dot(v, v))).
template <typename T>
constexpr tvec3<T> mix(const tvec3<T>& x, const tvec3<T>& y, T a)
{
    return x * (T(1) - a) + y * a;
}
template <typename T>
T smoothstep(T e0, T e1, T x)
{
    T t = (x - e0) / (e1 - e0);
    t = t < T(0) ? T(0) : (t > T(1) ? T(1) : t);
    return t * t * (T(3) - T(2) * t);
}
template <typename T>
tvec3<T> normalize(const tvec3<T>& v)
{
    return v * (T(1) / std::sqrt(v.x * v.x + v.y * v.y + v.z * v.z));
}

using vec2 = tvec2<float>;
using vec3 = tvec3<float>;
using vec4 = tvec4<float>;
using ivec2 = tvec2<std::int32_t>;
using ivec3 = tvec3<std::int32_t>;
using ivec4 = tvec4<std::int32_t>;
using uvec3 = tvec3<std::uint32_t>;

} // namespace glm
