// Headless frames of the resident worlds: one CUDA thread per pixel casts a ray
// through the voxel grid and shades the first visible face with the math of
// the reference's voxel pipeline (shaders/voxel.vert.hlsl:110-158,
// shaders/lighting.hlsl:3-30, shaders/mesh.frag.hlsl:12-82, shaders/fog.hlsl,
// shaders/projection.hlsl), writing RGBA8 sRGB pixels like its
// R8G8B8A8_SRGB render target (src/graphics/Renderer.cpp:42).
//
// A rasteriser with a depth test and no culling (src/graphics/Renderer.cpp:480-490)
// shows, per pixel centre, the nearest drawn face; the ray cast finds the same
// face: a face between cells A and B is drawn when one of them is an opaque
// block and the other is not (cells outside the region are air), and a torch
// is a 0.125 x 0.65 x 0.125 box without a bottom face
// (shaders/voxel.vert.hlsl:93-99, src/world/WorldGenerator.cu:221-303).
// Per-vertex values that are constant on a face (light, material) are exact;
// fog, interpolated per vertex there, is evaluated per pixel here.
#include "blk_internal.h"

#include <cmath>

namespace blk {
namespace {

struct RenderArgs {
    const uint8_t* ids;
    const uint8_t* light;
    const blk_render_params* params;
    int32_t W, H, D;
    const int4* origins; // [env] world coordinates of each env's local (0, 0, 0)
    uint64_t env_stride;
    uint32_t width, height, num_envs;
    uint8_t* out;     // RGBA8 (env, y, x, 4), or nullptr
    float* out_nchw;  // float32 (env, 3, y, x) = RGBA8 channel * (1 / 255), or nullptr
};

// Faces in the reference's order: left, right, top, bottom, front, back
// (-x, +x, +y, -y, +z, -z; src/world/Voxel.h:10-17).
enum : int { FaceLeft = 0, FaceRight, FaceTop, FaceBottom, FaceFront, FaceBack };
enum : int { MatGrassTop = 0, MatDirt = 1, MatStone = 2, MatGrassSide = 3, MatTorchSide = 6, MatTorchTop = 7 };

__device__ inline float fracf_(float x) { return x - floorf(x); }
__device__ inline float saturate_(float x) { return fminf(fmaxf(x, 0.0f), 1.0f); }
__device__ inline float lerp_(float a, float b, float t) { return a + t * (b - a); }

// shaders/mesh.frag.hlsl:12-17
__device__ inline float hash21(float px, float py)
{
    float p3x = fracf_(px * 0.1031f), p3y = fracf_(py * 0.1031f), p3z = fracf_(px * 0.1031f);
    const float d = p3x * (p3y + 33.33f) + p3y * (p3z + 33.33f) + p3z * (p3x + 33.33f);
    p3x += d;
    p3y += d;
    p3z += d;
    return fracf_((p3x + p3y) * p3z);
}

__device__ inline float srgb_to_linear(float c) { return powf(saturate_(c), 2.2f); }

// Linear albedo of a face texel (shaders/mesh.frag.hlsl:29-77).
__device__ void texel_color(int mat, float u, float v, float wx, float wz, float& r, float& g, float& b)
{
    float tx, ty;
    if (mat == MatGrassTop) {
        tx = floorf(wx * 16.0f);
        ty = floorf(wz * 16.0f);
    } else {
        tx = floorf(saturate_(u) * 15.999f);
        ty = floorf(saturate_(v) * 15.999f);
    }
    const float n = hash21(tx + static_cast<float>(mat) * 17.0f, ty + static_cast<float>(mat) * 17.0f);
    float cr, cg, cb;
    if (mat == MatGrassTop) {
        const float blade = hash21(tx * 1.7f + 4.0f, ty * 1.7f + 4.0f) >= 0.68f ? 1.0f : 0.0f;
        cr = lerp_(0.22f, 0.36f, n) + blade * 0.02f;
        cg = lerp_(0.50f, 0.64f, n) + blade * 0.04f;
        cb = lerp_(0.18f, 0.27f, n) + blade * 0.01f;
    } else if (mat == MatDirt) {
        cr = lerp_(0.35f, 0.56f, n);
        cg = lerp_(0.20f, 0.36f, n);
        cb = lerp_(0.10f, 0.18f, n);
    } else if (mat == MatStone) {
        cr = lerp_(0.43f, 0.57f, n);
        cg = lerp_(0.44f, 0.58f, n);
        cb = lerp_(0.44f, 0.58f, n);
    } else if (mat == MatGrassSide) {
        const float dr = lerp_(0.32f, 0.48f, n), dg = lerp_(0.20f, 0.31f, n), db = lerp_(0.11f, 0.17f, n);
        const float gr = lerp_(0.18f, 0.30f, n), gg = lerp_(0.46f, 0.58f, n), gb = lerp_(0.15f, 0.21f, n);
        float chance = 1.0f;
        if (ty >= 15.0f)
            chance = 0.0f;
        else if (ty >= 14.0f)
            chance = 0.12f;
        else if (ty >= 13.0f)
            chance = 0.32f;
        else if (ty >= 12.0f)
            chance = 0.58f;
        const float m = hash21(tx + 11.0f, ty + 11.0f) >= 1.0f - chance ? 1.0f : 0.0f;
        cr = lerp_(gr, dr, m);
        cg = lerp_(gg, dg, m);
        cb = lerp_(gb, db, m);
    } else if (mat == MatTorchSide) {
        const float e = v >= 0.72f ? 1.0f : 0.0f;
        cr = lerp_(lerp_(0.46f, 0.58f, n), lerp_(1.00f, 1.00f, n), e);
        cg = lerp_(lerp_(0.25f, 0.34f, n), lerp_(0.52f, 0.88f, n), e);
        cb = lerp_(lerp_(0.10f, 0.16f, n), lerp_(0.08f, 0.24f, n), e);
    } else { // torch top
        cr = lerp_(1.00f, 1.00f, n);
        cg = lerp_(0.52f, 0.88f, n);
        cb = lerp_(0.08f, 0.24f, n);
    }
    r = srgb_to_linear(cr);
    g = srgb_to_linear(cg);
    b = srgb_to_linear(cb);
}

// Component of a face normal along a direction (normals are axis unit vectors).
__device__ inline float face_dot(int face, float x, float y, float z)
{
    switch (face) {
    case FaceLeft: return -x;
    case FaceRight: return x;
    case FaceTop: return y;
    case FaceBottom: return -y;
    case FaceFront: return z;
    default: return -z;
    }
}

// shaders/lighting.hlsl:3-20
__device__ float face_sky_light(int face, const blk_render_params& p)
{
    const float* s = p.sky_light_direction;
    const float direct = lerp_(0.4f, 1.0f, saturate_(face_dot(face, s[0], s[1], s[2])));
    const float t = saturate_(s[1] / 0.6f);
    const float fallback = 1.0f - t * t * (3.0f - 2.0f * t);
    if (fallback < 1e-3f)
        return direct;
    const float k = rsqrtf(1.0f + 0.09f); // normalize(0, 1, 0.3)
    const float fl = lerp_(0.4f, 1.0f, saturate_(face_dot(face, 0.0f, k, 0.3f * k)));
    return lerp_(direct, fl, fallback);
}

// shaders/lighting.hlsl:22-30
__device__ float face_block_light(int face)
{
    const float ka = rsqrtf(0.35f * 0.35f + 0.85f * 0.85f + 0.45f * 0.45f);
    const float fa = rsqrtf(0.55f * 0.55f + 0.65f * 0.65f + 0.25f * 0.25f);
    const float key = saturate_(face_dot(face, 0.35f * ka, 0.85f * ka, 0.45f * ka));
    const float fill = saturate_(face_dot(face, -0.55f * fa, 0.65f * fa, -0.25f * fa));
    return 0.45f + key * 0.40f + fill * 0.15f;
}

// Texture coordinates of a point (lx, ly, lz in [0, 1] over the face's box)
// on a face, from the unit cube's vertex uvs (shaders/voxel.vert.hlsl:76-91).
__device__ inline void face_uv(int face, float lx, float ly, float lz, float& u, float& v)
{
    switch (face) {
    case FaceLeft:
    case FaceRight: u = lz; v = ly; break;
    case FaceTop: u = lx; v = lz; break;
    case FaceBottom: u = lz; v = lx; break;
    default: u = lx; v = ly; break;
    }
}

// shaders/voxel.vert.hlsl:48-58
__device__ inline int face_material(uint8_t block, int face)
{
    switch (block) {
    case Grass: return face == FaceTop ? MatGrassTop : (face == FaceBottom ? MatDirt : MatGrassSide);
    case Dirt: return MatDirt;
    case Stone: return MatStone;
    default: return face == FaceTop ? MatTorchTop : MatTorchSide;
    }
}

// Linear -> 8-bit sRGB as an sRGB render target stores it.
__device__ inline uint32_t to_srgb8(float c)
{
    c = saturate_(c);
    const float s = c <= 0.0031308f ? 12.92f * c : 1.055f * powf(c, 1.0f / 2.4f) - 0.055f;
    return static_cast<uint32_t>(__float2int_rn(s * 255.0f));
}

struct Hit {
    float s;        // ray parameter = view depth
    int face;
    uint8_t block;
    int cx, cy, cz; // cell of the voxel whose face was hit (local)
    int nx, ny, nz; // neighbour across the face, whose light the face shows (local)
    float lx, ly, lz; // hit point on the face box, [0, 1] per axis
};

__device__ inline bool in_region(const RenderArgs& a, int x, int y, int z)
{
    return x >= 0 && y >= 0 && z >= 0 && x < a.W && y < a.H && z < a.D;
}

__device__ inline uint8_t block_at(const RenderArgs& a, const uint8_t* ids, int x, int y, int z)
{
    return in_region(a, x, y, z) ? ids[(static_cast<uint64_t>(z) * a.W + x) * a.H + y] : Air;
}

__global__ void __launch_bounds__(128) render_kernel(RenderArgs a)
{
    const uint32_t env = blockIdx.y;
    const uint32_t pix = blockIdx.x * blockDim.x + threadIdx.x;
    if (env >= a.num_envs || pix >= a.width * a.height)
        return;
    const uint32_t px = pix % a.width, py = pix / a.width;
    const blk_render_params p = a.params[env];
    const uint8_t* ids = a.ids + static_cast<uint64_t>(env) * a.env_stride;
    const uint8_t* lt = a.light + static_cast<uint64_t>(env) * a.env_stride;

    // Ray through the pixel centre (shaders/projection.hlsl:22-35): the view
    // direction has forward component 1, so the ray parameter is view depth.
    const float t = tanf(p.fov_radians * 0.5f);
    const float aspect = static_cast<float>(a.width) / static_cast<float>(a.height);
    const float xn = (static_cast<float>(px) + 0.5f) / static_cast<float>(a.width) * 2.0f - 1.0f;
    const float yn = (static_cast<float>(py) + 0.5f) / static_cast<float>(a.height) * 2.0f - 1.0f;
    const float vx = xn * aspect * t, vy = -yn * t;
    const float d[3] = { p.right[0] * vx + p.up[0] * vy + p.forward[0], p.right[1] * vx + p.up[1] * vy + p.forward[1],
        p.right[2] * vx + p.up[2] * vy + p.forward[2] };
    // Local coordinates: region cell (0, 0, 0) spans [0, 1)^3.
    const int4 org = a.origins[env];
    const float o[3] = { p.origin[0] - org.x, p.origin[1] - org.y, p.origin[2] - org.z };
    const int dims[3] = { a.W, a.H, a.D };
    constexpr float kNear = 0.05f;
    // Past the fog end a face takes the sky colour (fog factor 1), which is
    // also the colour of an empty pixel: the walk stops there.
    const float far = p.fog_end > p.fog_start ? fminf(p.far_plane, p.fog_end) : p.far_plane;

    // Parameter range of the ray inside the region box, and the axis whose
    // boundary it enters through when the camera is outside.
    float s0 = 0.0f, s1 = far;
    int entry_axis = -1;
    for (int k = 0; k < 3; ++k) {
        if (fabsf(d[k]) < 1e-20f) {
            if (o[k] < 0.0f || o[k] >= static_cast<float>(dims[k]))
                s1 = -1.0f;
        } else {
            float ta = (0.0f - o[k]) / d[k], tb = (static_cast<float>(dims[k]) - o[k]) / d[k];
            if (ta > tb) {
                const float tmp = ta;
                ta = tb;
                tb = tmp;
            }
            if (ta > s0) {
                s0 = ta;
                entry_axis = k;
            }
            s1 = fminf(s1, tb);
        }
    }

    Hit hit;
    hit.s = -1.0f;
    // Face of opaque cell `owner` towards the non-opaque cell `other` (adjacent
    // along axis ax), hit at ray parameter sh.
    auto face_hit = [&](const int* owner, const int* other, int ax, float sh) {
        const int dir = other[ax] - owner[ax];
        hit.s = sh;
        hit.face = ax == 0 ? (dir > 0 ? FaceRight : FaceLeft)
                           : (ax == 1 ? (dir > 0 ? FaceTop : FaceBottom) : (dir > 0 ? FaceFront : FaceBack));
        hit.block = block_at(a, ids, owner[0], owner[1], owner[2]);
        hit.cx = owner[0];
        hit.cy = owner[1];
        hit.cz = owner[2];
        hit.nx = other[0];
        hit.ny = other[1];
        hit.nz = other[2];
        hit.lx = saturate_(o[0] + d[0] * sh - owner[0]);
        hit.ly = saturate_(o[1] + d[1] * sh - owner[1]);
        hit.lz = saturate_(o[2] + d[2] * sh - owner[2]);
        if (ax == 0)
            hit.lx = dir > 0 ? 1.0f : 0.0f;
        else if (ax == 1)
            hit.ly = dir > 0 ? 1.0f : 0.0f;
        else
            hit.lz = dir > 0 ? 1.0f : 0.0f;
    };
    if (s0 <= s1) {
        // Amanatides-Woo traversal from the entry point.
        int c[3], st[3];
        float tmax[3], tdel[3];
        for (int k = 0; k < 3; ++k) {
            const float e = o[k] + d[k] * s0;
            int ck = static_cast<int>(floorf(e));
            ck = min(max(ck, 0), dims[k] - 1);
            c[k] = ck;
            if (d[k] > 0.0f) {
                st[k] = 1;
                tdel[k] = 1.0f / d[k];
                tmax[k] = (static_cast<float>(ck + 1) - o[k]) / d[k];
            } else if (d[k] < 0.0f) {
                st[k] = -1;
                tdel[k] = -1.0f / d[k];
                tmax[k] = (static_cast<float>(ck) - o[k]) / d[k];
            } else {
                st[k] = 0;
                tdel[k] = 3.0e38f;
                tmax[k] = 3.0e38f;
            }
        }
        float s_cell = s0; // where the ray entered the current cell
        // Entering from outside the region (air) into an opaque boundary cell.
        if (entry_axis >= 0 && s0 >= kNear && s0 <= far && is_opaque(block_at(a, ids, c[0], c[1], c[2]))) {
            int outside[3] = { c[0], c[1], c[2] };
            outside[entry_axis] -= st[entry_axis];
            face_hit(c, outside, entry_axis, s0);
        }
        const int max_steps = a.W + a.H + a.D + 3;
        for (int it = 0; it < max_steps && hit.s < 0.0f; ++it) {
            const uint8_t cur = block_at(a, ids, c[0], c[1], c[2]);
            const int ax = tmax[0] <= tmax[1] ? (tmax[0] <= tmax[2] ? 0 : 2) : (tmax[1] <= tmax[2] ? 1 : 2);
            const float s_cross = tmax[ax];
            if (cur == Torch) {
                // The torch box inside the cell: entry (or, through the missing
                // bottom or from inside, exit) face within this cell's span.
                const float lo[3] = { c[0] + 0.4375f, static_cast<float>(c[1]), c[2] + 0.4375f };
                const float hi[3] = { c[0] + 0.5625f, c[1] + 0.65f, c[2] + 0.5625f };
                float tin = -3.0e38f, tout = 3.0e38f;
                int fin = -1, fout = -1;
                for (int k = 0; k < 3; ++k) {
                    if (d[k] == 0.0f) {
                        if (o[k] < lo[k] || o[k] > hi[k])
                            tin = 3.0e38f;
                        continue;
                    }
                    float ta = (lo[k] - o[k]) / d[k], tb = (hi[k] - o[k]) / d[k];
                    // faces: k = 0 -> left (lo) / right (hi); k = 1 -> bottom / top; k = 2 -> back / front
                    int fa = k == 0 ? FaceLeft : (k == 1 ? FaceBottom : FaceBack);
                    int fb = k == 0 ? FaceRight : (k == 1 ? FaceTop : FaceFront);
                    if (ta > tb) {
                        const float tmp = ta;
                        ta = tb;
                        tb = tmp;
                        const int f = fa;
                        fa = fb;
                        fb = f;
                    }
                    if (ta > tin) {
                        tin = ta;
                        fin = fa;
                    }
                    if (tb < tout) {
                        tout = tb;
                        fout = fb;
                    }
                }
                const float lo_s = fmaxf(s_cell, kNear);
                if (tin <= tout) {
                    float sh = -1.0f;
                    int fh = -1;
                    if (fin >= 0 && fin != FaceBottom && tin >= lo_s && tin <= s_cross)
                        sh = tin, fh = fin;
                    else if (fout >= 0 && fout != FaceBottom && tout >= lo_s && tout <= s_cross)
                        sh = tout, fh = fout;
                    if (fh >= 0 && sh <= far) {
                        hit.s = sh;
                        hit.face = fh;
                        hit.block = Torch;
                        hit.cx = c[0];
                        hit.cy = c[1];
                        hit.cz = c[2];
                        const int off[6][3] = { { -1, 0, 0 }, { 1, 0, 0 }, { 0, 1, 0 }, { 0, -1, 0 }, { 0, 0, 1 },
                            { 0, 0, -1 } };
                        hit.nx = c[0] + off[fh][0];
                        hit.ny = c[1] + off[fh][1];
                        hit.nz = c[2] + off[fh][2];
                        const float q[3] = { o[0] + d[0] * sh, o[1] + d[1] * sh, o[2] + d[2] * sh };
                        hit.lx = saturate_((q[0] - lo[0]) / 0.125f);
                        hit.ly = saturate_((q[1] - lo[1]) / 0.65f);
                        hit.lz = saturate_((q[2] - lo[2]) / 0.125f);
                        break;
                    }
                }
            }
            if (s_cross > s1 + 1e-4f || s_cross > far)
                break;
            int nxt[3] = { c[0], c[1], c[2] };
            nxt[ax] += st[ax];
            const uint8_t nb = block_at(a, ids, nxt[0], nxt[1], nxt[2]);
            const bool cur_op = is_opaque(cur), nb_op = is_opaque(nb);
            if (s_cross >= kNear && cur_op != nb_op) {
                // The opaque one of the two cells owns the drawn face.
                if (cur_op)
                    face_hit(c, nxt, ax, s_cross);
                else
                    face_hit(nxt, c, ax, s_cross);
                break;
            }
            c[0] = nxt[0];
            c[1] = nxt[1];
            c[2] = nxt[2];
            s_cell = s_cross;
            tmax[ax] += tdel[ax];
            if (!in_region(a, c[0], c[1], c[2]))
                break;
        }
    }

    float r, g, b;
    if (hit.s < 0.0f) {
        r = p.sky_color[0];
        g = p.sky_color[1];
        b = p.sky_color[2];
    } else {
        // Face light: the neighbour's levels, a torch shows block light 15
        // (src/world/WorldGenerator.cu:246-262, shaders/voxel.vert.hlsl:131-153).
        uint32_t sky = 0, blk = 0;
        if (in_region(a, hit.nx, hit.ny, hit.nz)) {
            const uint8_t l = lt[(static_cast<uint64_t>(hit.nz) * a.W + hit.nx) * a.H + hit.ny];
            sky = l >> 4;
            blk = l & 15u;
        }
        if (hit.block == Torch)
            blk = 15;
        const uint32_t cur_sky = sky - min(sky, p.sky_light_dimming);
        const float light = fmaxf(static_cast<float>(cur_sky) * face_sky_light(hit.face, p),
                                static_cast<float>(blk) * face_block_light(hit.face))
            / 15.0f;
        float u, v;
        face_uv(hit.face, hit.lx, hit.ly, hit.lz, u, v);
        const float wx = o[0] + d[0] * hit.s + org.x, wz = o[2] + d[2] * hit.s + org.z;
        float ar, ag, ab;
        texel_color(face_material(hit.block, hit.face), u, v, wx, wz, ar, ag, ab);
        const float fog = saturate_((hit.s - p.fog_start) / fmaxf(p.fog_end - p.fog_start, 0.001f));
        r = lerp_(saturate_(ar * light), p.sky_color[0], fog);
        g = lerp_(saturate_(ag * light), p.sky_color[1], fog);
        b = lerp_(saturate_(ab * light), p.sky_color[2], fog);
    }
    const uint32_t cr = to_srgb8(r), cg = to_srgb8(g), cb = to_srgb8(b);
    if (a.out)
        reinterpret_cast<uint32_t*>(a.out)[(static_cast<uint64_t>(env) * a.height + py) * a.width + px]
            = cr | (cg << 8) | (cb << 16) | (255u << 24);
    if (a.out_nchw) {
        // The observation conversion of the same bytes (src/environment/CudaObservation.cu:13-31).
        const uint64_t plane = static_cast<uint64_t>(a.width) * a.height;
        float* o = a.out_nchw + static_cast<uint64_t>(env) * 3 * plane + static_cast<uint64_t>(py) * a.width + px;
        const float k = 1.0f / 255.0f;
        o[0] = __fmul_rn(static_cast<float>(cr), k);
        o[plane] = __fmul_rn(static_cast<float>(cg), k);
        o[2 * plane] = __fmul_rn(static_cast<float>(cb), k);
    }
}

} // namespace

int launch_render(blk_ctx* ctx, const blk_render_params* params, uint32_t width, uint32_t height, uint8_t* out,
    float* out_nchw, cudaStream_t stream)
{
    RenderArgs a;
    a.ids = ctx->ids;
    a.light = ctx->light;
    a.params = params;
    a.W = static_cast<int32_t>(ctx->cfg.width);
    a.H = static_cast<int32_t>(ctx->cfg.height);
    a.D = static_cast<int32_t>(ctx->cfg.depth);
    a.origins = ctx->origins;
    a.env_stride = ctx->env_stride;
    a.width = width;
    a.height = height;
    a.num_envs = ctx->cfg.num_envs;
    a.out = out;
    a.out_nchw = out_nchw;
    const dim3 grid((width * height + 127) / 128, ctx->cfg.num_envs);
    render_kernel<<<grid, 128, 0, stream>>>(a);
    return cuda_fail(cudaGetLastError(), "render_kernel launch");
}

} // namespace blk
