// C entry points over the reference's sky functions (src/world/Lighting.cpp),
// compiled from the reference sources into oracle/_ref/libref_lighting.so.
// Test infrastructure only; never linked into the product library.
#include <world/Lighting.h>

#include <cstdint>

extern "C" {

std::uint8_t ref_sky_light_at(std::uint32_t t) { return blocklab::skyLightAtTime(static_cast<blocklab::WorldTime>(t)); }

void ref_sky_color_at(std::uint32_t t, float* out)
{
    const blocklab::Vec3 c = blocklab::skyColorAtTime(static_cast<blocklab::WorldTime>(t));
    out[0] = c.x;
    out[1] = c.y;
    out[2] = c.z;
}

void ref_sky_direction_at(std::uint32_t t, float* out)
{
    const blocklab::Vec3 d = blocklab::skyLightDirectionAtTime(static_cast<blocklab::WorldTime>(t));
    out[0] = d.x;
    out[1] = d.y;
    out[2] = d.z;
}
}
