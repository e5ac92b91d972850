// Device loader for 3DGS .ply scenes (splax/io.py:78-98, load_ply): the header is parsed on the
// host, the vertex records stream through two pinned buffers and two device staging buffers
// (disk read of chunk k+1 overlaps the copy and decode of chunk k), and one kernel per chunk
// decodes each record into the five render-space arrays:
//   means = (x, y, z), scales = exp(scale_0..2), quats = rot_0..3 / |rot| (wxyz, as stored),
//   colors = clip(f_dc * C0 + 0.5, 0, 1) with C0 the degree-0 SH constant,
//   opacities = sigmoid(opacity).
// Only binary little-endian files whose first element is `vertex` with scalar properties are
// read (the format 3DGS tools and the reference's write_ply produce); the needed fields must be
// float32, other properties of any scalar type are skipped by their sizes.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "kernels.h"

namespace splax {
namespace {

constexpr float kShC0 = 0.28209479177387814f;
constexpr int kPlyThreads = 256;

__device__ __forceinline__ float load_f32(const unsigned char* p, bool aligned) {
  if (aligned) return *reinterpret_cast<const float*>(p);
  uint32_t u = static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
               (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
  return __uint_as_float(u);
}

__global__ void __launch_bounds__(kPlyThreads)
ply_decode_kernel(const unsigned char* __restrict__ body, int64_t count, PlyLayout L,
                  int64_t first, float* means, float* scales, float* quats, float* colors,
                  float* opacities) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kPlyThreads + threadIdx.x;
  if (i >= count) return;
  const unsigned char* r = body + i * L.stride;
  const bool al = L.aligned;
  const int64_t v = first + i;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    means[3 * v + k] = load_f32(r + L.off[k], al);
    scales[3 * v + k] = expf(load_f32(r + L.off[3 + k], al));
    colors[3 * v + k] = fminf(fmaxf(fmaf(load_f32(r + L.off[10 + k], al), kShC0, 0.5f), 0.0f), 1.0f);
  }
  float q[4], ss = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    q[k] = load_f32(r + L.off[6 + k], al);
    ss = fmaf(q[k], q[k], ss);
  }
  const float nrm = sqrtf(ss);
#pragma unroll
  for (int k = 0; k < 4; ++k) quats[4 * v + k] = q[k] / nrm;
  opacities[v] = 1.0f / (1.0f + expf(-load_f32(r + L.off[13], al)));
}

int type_size(const std::string& t) {
  if (t == "char" || t == "uchar" || t == "int8" || t == "uint8") return 1;
  if (t == "short" || t == "ushort" || t == "int16" || t == "uint16") return 2;
  if (t == "int" || t == "uint" || t == "float" || t == "int32" || t == "uint32" ||
      t == "float32")
    return 4;
  if (t == "double" || t == "float64") return 8;
  return -1;
}

}  // namespace

// Needed fields in PlyLayout::off order.
static const char* const kPlyFields[14] = {"x", "y", "z", "scale_0", "scale_1", "scale_2",
                                           "rot_0", "rot_1", "rot_2", "rot_3", "f_dc_0",
                                           "f_dc_1", "f_dc_2", "opacity"};

int ply_parse_header(FILE* f, PlyLayout* L, int64_t* count, int64_t* body_offset,
                     std::string* why) {
  char line[1024];
  auto next = [&](void) -> bool {
    if (!std::fgets(line, sizeof line, f)) return false;
    size_t n = std::strlen(line);
    while (n && (line[n - 1] == '\n' || line[n - 1] == '\r')) line[--n] = '\0';
    return true;
  };
  if (!next() || std::strcmp(line, "ply") != 0) {
    *why = "not a PLY file";
    return -1;
  }
  bool fmt = false, in_vertex = false, seen_vertex = false;
  int64_t n = -1, stride = 0;
  int found = 0;
  for (int k = 0; k < 14; ++k) L->off[k] = -1;
  while (true) {
    if (!next()) {
      *why = "header ends before end_header";
      return -1;
    }
    char a[64] = {0}, b[64] = {0}, c[256] = {0};
    const int toks = std::sscanf(line, "%63s %63s %255s", a, b, c);
    if (toks <= 0) continue;
    const std::string w0 = a;
    if (w0 == "end_header") break;
    if (w0 == "comment" || w0 == "obj_info") continue;
    if (w0 == "format") {
      if (std::string(b) != "binary_little_endian") {
        *why = std::string("unsupported PLY format ") + b + " (binary_little_endian only)";
        return -1;
      }
      fmt = true;
    } else if (w0 == "element") {
      if (seen_vertex) {
        in_vertex = false;  // later elements are not read
        continue;
      }
      if (std::string(b) != "vertex") {
        *why = "the first PLY element must be 'vertex'";
        return -1;
      }
      seen_vertex = in_vertex = true;
      n = std::atoll(c);
    } else if (w0 == "property") {
      if (!in_vertex) continue;
      if (std::string(b) == "list") {
        *why = "list properties in the vertex element are not supported";
        return -1;
      }
      const int sz = type_size(b);
      if (sz < 0) {
        *why = std::string("unknown PLY property type ") + b;
        return -1;
      }
      for (int k = 0; k < 14; ++k) {
        if (std::string(c) == kPlyFields[k]) {
          if (sz != 4 || !(std::string(b) == "float" || std::string(b) == "float32")) {
            *why = std::string("PLY field ") + c + " must be float32";
            return -1;
          }
          if (L->off[k] < 0) ++found;
          L->off[k] = static_cast<int32_t>(stride);
        }
      }
      stride += sz;
    }
  }
  if (!fmt || !seen_vertex || n < 0) {
    *why = "PLY header lacks the format or the vertex element";
    return -1;
  }
  if (found != 14) {
    for (int k = 0; k < 14; ++k)
      if (L->off[k] < 0) {
        *why = std::string("PLY vertex element lacks the field ") + kPlyFields[k];
        break;
      }
    return -1;
  }
  L->stride = stride;
  bool al = stride % 4 == 0;
  for (int k = 0; k < 14; ++k) al = al && L->off[k] % 4 == 0;
  L->aligned = al;
  *count = n;
  *body_offset = std::ftell(f);
  return 0;
}

void launch_ply_decode(const unsigned char* body, int64_t count, const PlyLayout& L,
                       int64_t first, float* means, float* scales, float* quats, float* colors,
                       float* opacities, cudaStream_t stream) {
  if (count <= 0) return;
  const int64_t blocks = (count + kPlyThreads - 1) / kPlyThreads;
  ply_decode_kernel<<<static_cast<unsigned>(blocks), kPlyThreads, 0, stream>>>(
      body, count, L, first, means, scales, quats, colors, opacities);
}

}  // namespace splax
