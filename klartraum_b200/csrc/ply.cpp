// Reader of 3D Gaussian Splatting .ply files, the input of klartraum's loadPLYModel
// (src/vulkan_gaussian_splatting.cpp:367-417), which reads them through spz::loadSplatFromPly.
//
// The file: an ASCII header ("ply", "format binary_little_endian 1.0" or "format ascii 1.0",
// "element vertex N", one "property <type> <name>" line per attribute, "end_header"), then N
// vertices. The attributes used are x y z, f_dc_0..2, f_rest_0..44 (channel-major: 15 per channel
// for degree 3), opacity (logit), scale_0..2 (log), rot_0..3 (w, x, y, z). loadPLYModel then keeps
// the Gaussians inside the box [-1.5, 1.5]^3, applies alpha = sigmoid(opacity) and scale = exp,
// and stores the colour pre-baked as 0.5 + 0.282095 dc (it does not copy the higher SH
// coefficients; they are zero here). Quaternions are stored (x, y, z, w) as given, not normalised.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "kt_gs.h"

namespace {

enum class PType { I8, U8, I16, U16, I32, U32, F32, F64, Bad };

PType ptype(const std::string& t) {
    if (t == "char" || t == "int8") return PType::I8;
    if (t == "uchar" || t == "uint8") return PType::U8;
    if (t == "short" || t == "int16") return PType::I16;
    if (t == "ushort" || t == "uint16") return PType::U16;
    if (t == "int" || t == "int32") return PType::I32;
    if (t == "uint" || t == "uint32") return PType::U32;
    if (t == "float" || t == "float32") return PType::F32;
    if (t == "double" || t == "float64") return PType::F64;
    return PType::Bad;
}

size_t psize(PType t) {
    switch (t) {
        case PType::I8: case PType::U8: return 1;
        case PType::I16: case PType::U16: return 2;
        case PType::I32: case PType::U32: case PType::F32: return 4;
        case PType::F64: return 8;
        default: return 0;
    }
}

double pread(const uint8_t* p, PType t) {
    switch (t) {
        case PType::I8: { int8_t v; std::memcpy(&v, p, 1); return v; }
        case PType::U8: return p[0];
        case PType::I16: { int16_t v; std::memcpy(&v, p, 2); return v; }
        case PType::U16: { uint16_t v; std::memcpy(&v, p, 2); return v; }
        case PType::I32: { int32_t v; std::memcpy(&v, p, 4); return v; }
        case PType::U32: { uint32_t v; std::memcpy(&v, p, 4); return v; }
        case PType::F32: { float v; std::memcpy(&v, p, 4); return v; }
        case PType::F64: { double v; std::memcpy(&v, p, 8); return v; }
        default: return 0.0;
    }
}

double sigmoid(double x) { return 1.0 / (1.0 + std::exp(-x)); }

struct Prop {
    std::string name;
    PType type;
    size_t offset;
};

}  // namespace

extern "C" kt_status kt_gs_ply_decode(const char* path, kt_gaussian3d* out, uint64_t capacity, uint64_t* count) {
    if (!path || !count) return KT_ERR_ARG;
    std::ifstream f(path, std::ios::binary);
    if (!f) return KT_ERR_IO;
    std::string line;
    if (!std::getline(f, line) || line.rfind("ply", 0) != 0) return KT_ERR_IO;
    bool binary = false, ascii = false, in_vertex = false;
    uint64_t nv = 0;
    std::vector<Prop> props;
    size_t stride = 0;
    for (;;) {
        if (!std::getline(f, line)) return KT_ERR_IO;
        if (!line.empty() && line.back() == '\r') line.pop_back();
        std::istringstream ls(line);
        std::string w;
        ls >> w;
        if (w == "format") {
            std::string fmt;
            ls >> fmt;
            binary = fmt == "binary_little_endian";
            ascii = fmt == "ascii";
        } else if (w == "element") {
            std::string name;
            uint64_t cnt = 0;
            ls >> name >> cnt;
            if (in_vertex && name != "vertex") in_vertex = false;
            if (name == "vertex") {
                in_vertex = true;
                nv = cnt;
            } else if (nv == 0 && cnt > 0) {
                return KT_ERR_IO;  // elements before the vertices are not supported
            }
        } else if (w == "property" && in_vertex) {
            std::string t, name;
            ls >> t;
            if (t == "list") return KT_ERR_IO;
            ls >> name;
            const PType pt = ptype(t);
            if (pt == PType::Bad) return KT_ERR_IO;
            props.push_back({name, pt, stride});
            stride += psize(pt);
        } else if (w == "end_header") {
            break;
        }
    }
    if (!(binary || ascii) || nv > (1ull << 32)) return KT_ERR_IO;
    if (nv == 0) {
        *count = 0;
        return KT_OK;
    }
    auto find = [&](const std::string& n) -> int {
        for (size_t i = 0; i < props.size(); ++i)
            if (props[i].name == n) return (int)i;
        return -1;
    };
    const char* need[] = {"x", "y", "z", "f_dc_0", "f_dc_1", "f_dc_2", "opacity", "scale_0", "scale_1", "scale_2",
                          "rot_0", "rot_1", "rot_2", "rot_3"};
    int idx[14];
    for (int i = 0; i < 14; ++i)
        if ((idx[i] = find(need[i])) < 0) return KT_ERR_IO;

    std::vector<double> v(props.size());
    std::vector<uint8_t> rec(stride);
    uint64_t kept = 0;
    for (uint64_t i = 0; i < nv; ++i) {
        if (binary) {
            if (!f.read(reinterpret_cast<char*>(rec.data()), (std::streamsize)stride)) return KT_ERR_IO;
            for (size_t k = 0; k < props.size(); ++k) v[k] = pread(rec.data() + props[k].offset, props[k].type);
        } else {
            for (size_t k = 0; k < props.size(); ++k)
                if (!(f >> v[k])) return KT_ERR_IO;
        }
        const float x = (float)v[idx[0]], y = (float)v[idx[1]], z = (float)v[idx[2]];
        const float clip = 1.5f;  // loadPLYModel's clip box
        if (x < -clip || x > clip || y < -clip || y > clip || z < -clip || z > clip) continue;
        if (out) {
            if (kept >= capacity) return KT_ERR_CAPACITY;
            kt_gaussian3d& g = out[kept];
            std::memset(&g, 0, sizeof(g));
            g.position[0] = x;
            g.position[1] = y;
            g.position[2] = z;
            g.rotation[0] = (float)v[idx[11]];  // rot_1 .. rot_3 = x, y, z; rot_0 = w
            g.rotation[1] = (float)v[idx[12]];
            g.rotation[2] = (float)v[idx[13]];
            g.rotation[3] = (float)v[idx[10]];
            g.alpha = (float)sigmoid((double)(float)v[idx[6]]);
            for (int c = 0; c < 3; ++c) {
                const float dc = (float)v[idx[3 + c]];
                g.color[c] = (float)(0.5 + 0.282095 * (double)dc);
                g.scale[c] = std::exp((float)v[idx[7 + c]]);
            }
        }
        ++kept;
    }
    *count = kept;
    return KT_OK;
}
