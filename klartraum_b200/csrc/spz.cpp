// Reader of .spz Gaussian files (the format of nianticlabs/spz, which klartraum's loadSPZModel
// reads through spz::loadSpzPacked + PackedGaussians::unpack, src/vulkan_gaussian_splatting.cpp:322-365).
//
// The library is not vendored in the reference (3rdparty/spz is an empty submodule), so the
// format is restated from its published description:
//   gzip stream of
//     header (16 bytes, little endian): magic 0x5053474e ("NGSP"), version (1..3), point count,
//       SH degree (u8, 0..3), fractional bits (u8), flags (u8; bit 0 = antialiased), reserved (u8)
//     positions  v1: 3 half floats per point; v2+: 3 x 24-bit signed fixed point, value / 2^fractional_bits
//     alphas     1 byte per point: sigmoid(opacity) * 255
//     colours    3 bytes per point: (dc * 0.15 + 0.5) * 255, dc = the degree-0 SH coefficient
//     scales     3 bytes per point: (log scale + 10) * 16
//     rotations  v1/v2: 3 bytes per point, x, y, z of the unit quaternion as (v + 1) * 127.5, w >= 0
//                recovered from the norm; v3: 4 bytes, the index of the largest component (2 bits)
//                and the other three as 9-bit magnitudes over sqrt(1/2) with a sign bit each
//     SH         per point, (d+1)^2 - 1 coefficients x 3 channels, each (v * 128 + 128) bytes,
//                coefficient-major (R, G, B of coefficient 1, then of coefficient 2, ...)
// loadSPZModel then applies alpha = sigmoid(logit) and scale = exp(log scale) and keeps the colour
// as the raw DC coefficient (the shader adds 0.5 + 0.282095 dc); the coordinate converter it
// passes is the identity. Coefficients above the file's degree are zero here.
#include <zlib.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "kt_gs.h"

namespace {

constexpr uint32_t kSpzMagic = 0x5053474eu;
constexpr uint64_t kSpzMaxPoints = 1ull << 31;  // keeps every per-point size below 2^40

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            bits = sign | (uint32_t)(112 - e) << 23 | (m & 0x3FFu) << 13;
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | man << 13;
    } else {
        bits = sign | (exp + 112) << 23 | man << 13;
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

double sigmoid(double x) { return 1.0 / (1.0 + std::exp(-x)); }

bool read_all(const char* path, std::vector<uint8_t>& out, std::string& err) {
    gzFile f = gzopen(path, "rb");
    if (!f) {
        err = std::string("cannot open ") + path;
        return false;
    }
    uint8_t buf[1 << 16];
    for (;;) {
        const int got = gzread(f, buf, sizeof(buf));
        if (got < 0) {
            int code = 0;
            err = std::string("gzip read failed: ") + gzerror(f, &code);
            gzclose(f);
            return false;
        }
        if (got == 0) break;
        out.insert(out.end(), buf, buf + got);
    }
    gzclose(f);
    return true;
}

}  // namespace

extern "C" kt_status kt_gs_spz_decode(const char* path, kt_gaussian3d* out, uint64_t capacity, uint64_t* count,
                                      uint32_t* sh_degree) {
    if (!path || !count) return KT_ERR_ARG;
    std::vector<uint8_t> d;
    std::string err;
    if (!read_all(path, d, err)) return KT_ERR_IO;
    if (d.size() < 16) return KT_ERR_IO;
    uint32_t magic, version, npts;
    std::memcpy(&magic, d.data(), 4);
    std::memcpy(&version, d.data() + 4, 4);
    std::memcpy(&npts, d.data() + 8, 4);
    const uint32_t deg = d[12], frac = d[13];
    if (magic != kSpzMagic || version < 1 || version > 3 || deg > 3 || frac > 30 || npts > kSpzMaxPoints)
        return KT_ERR_IO;
    const uint64_t n = npts;
    const uint32_t sh_dim = (deg + 1) * (deg + 1) - 1;
    const uint64_t pos_b = version == 1 ? n * 6 : n * 9;
    const uint64_t rot_b = version == 3 ? n * 4 : n * 3;
    const uint64_t need = 16 + pos_b + n + n * 3 + n * 3 + rot_b + n * sh_dim * 3;
    if (d.size() < need) return KT_ERR_IO;
    *count = n;
    if (sh_degree) *sh_degree = deg;
    if (!out) return KT_OK;  // size query
    if (capacity < n) return KT_ERR_CAPACITY;

    const uint8_t* p_pos = d.data() + 16;
    const uint8_t* p_alpha = p_pos + pos_b;
    const uint8_t* p_col = p_alpha + n;
    const uint8_t* p_scale = p_col + n * 3;
    const uint8_t* p_rot = p_scale + n * 3;
    const uint8_t* p_sh = p_rot + rot_b;
    const float fscale = 1.0f / (float)(1u << frac);
    for (uint64_t i = 0; i < n; ++i) {
        kt_gaussian3d& g = out[i];
        std::memset(&g, 0, sizeof(g));
        for (int j = 0; j < 3; ++j) {
            if (version == 1) {
                uint16_t h;
                std::memcpy(&h, p_pos + i * 6 + j * 2, 2);
                g.position[j] = half_to_float(h);
            } else {
                const uint8_t* b = p_pos + i * 9 + j * 3;
                int32_t v = (int32_t)((uint32_t)b[0] | (uint32_t)b[1] << 8 | (uint32_t)b[2] << 16);
                if (v & 0x800000) v |= (int32_t)0xFF000000u;  // sign of the 24-bit value
                g.position[j] = (float)v * fscale;
            }
        }
        // scale: exp of the stored log scale (loadSPZModel's activation)
        for (int j = 0; j < 3; ++j) g.scale[j] = std::exp((float)p_scale[i * 3 + j] / 16.0f - 10.0f);
        if (version == 3) {
            const uint8_t* r = p_rot + i * 4;
            uint32_t comp = (uint32_t)r[0] | (uint32_t)r[1] << 8 | (uint32_t)r[2] << 16 | (uint32_t)r[3] << 24;
            const uint32_t mask = (1u << 9) - 1u;
            const int largest = (int)(comp >> 30);
            float q[4] = {0, 0, 0, 0}, ss = 0.0f;
            for (int k = 3; k >= 0; --k) {
                if (k == largest) continue;
                const uint32_t mag = comp & mask, neg = (comp >> 9) & 1u;
                comp >>= 10;
                float v = 0.70710678118654752f * (float)mag / (float)mask;
                if (neg) v = -v;
                q[k] = v;
                ss += v * v;
            }
            q[largest] = std::sqrt(std::fmax(0.0f, 1.0f - ss));
            for (int k = 0; k < 4; ++k) g.rotation[k] = q[k];
        } else {
            const uint8_t* r = p_rot + i * 3;
            float ss = 0.0f;
            for (int k = 0; k < 3; ++k) {
                g.rotation[k] = (float)r[k] / 127.5f - 1.0f;
                ss += g.rotation[k] * g.rotation[k];
            }
            g.rotation[3] = std::sqrt(std::fmax(0.0f, 1.0f - ss));
        }
        // alpha: the stored sigmoid, back to the logit and through the reference's double sigmoid
        const float a = (float)p_alpha[i] / 255.0f;
        const float logit = std::log(a / (1.0f - a));
        g.alpha = (float)sigmoid((double)logit);
        for (int j = 0; j < 3; ++j) g.color[j] = ((float)p_col[i * 3 + j] / 255.0f - 0.5f) / 0.15f;
        const uint8_t* s = p_sh + i * sh_dim * 3;
        for (uint32_t k = 0; k < sh_dim; ++k) {
            g.shR[k] = ((float)s[k * 3 + 0] - 128.0f) / 128.0f;
            g.shG[k] = ((float)s[k * 3 + 1] - 128.0f) / 128.0f;
            g.shB[k] = ((float)s[k * 3 + 2] - 128.0f) / 128.0f;
        }
    }
    return KT_OK;
}
