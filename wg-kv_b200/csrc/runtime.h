#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wgkv {

// Encode a 2D bf16 tensor map: `inner` contiguous elements per row, `outer`
// rows `row_stride_elems` apart, box {box_inner, box_outer}.
bool encode_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                    uint32_t box_inner, uint32_t box_outer, bool swizzle128);

// Encode a 3D bf16 tensor map: dims[0] contiguous elements, dims[1] and dims[2] `stride_elems[0]`
// and `stride_elems[1]` elements apart, box {box[0], box[1], box[2]} (lands as box[1] * box[2] rows
// of box[0] elements, dimension 1 fastest).
bool encode_3d_bf16(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t stride_elems[2],
                    const uint32_t box[3], bool swizzle128);

// SM count of the current device (cached), -1 on error.
int device_sms();

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace wgkv
