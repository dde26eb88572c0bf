// Float RGB image -> 8-bit layouts (HWC RGB, HWC RGBA with alpha 255, planar
// CHW RGB) for sm_100a: csrc/nodes/img_layout.cu:9-115 of the reference.
//
// Each channel becomes (uint8)(saturate(x) * 255), truncating (NaN -> 0).
// HBM-bound byte work: 12 bytes read per pixel and 3 or 4 written.  Each
// thread converts four pixels with three 16-byte loads and one 16-byte
// (RGBA), three 4-byte (RGB) or three 4-byte planar (CHW) stores, so every
// access is a full, coalesced vector; the last n % 4 pixels, and inputs whose
// pointers are not aligned for that, go through a one-pixel-per-thread kernel.
#include "common.cuh"

namespace xsg {

constexpr int kImgThreads = 256;

__device__ __forceinline__ uint32_t to_byte(float x) {
    return static_cast<uint32_t>(static_cast<unsigned char>(__saturatef(x) * 255.0f));
}

template <int kLayout>
__global__ void __launch_bounds__(kImgThreads)
    image_bytes_vec_kernel(const float4* __restrict__ in, int64_t n_quads, int64_t n_pixels,
                           uint8_t* __restrict__ out) {
    for (int64_t q = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; q < n_quads;
         q += int64_t(gridDim.x) * blockDim.x) {
        const float4 a = in[3 * q], b = in[3 * q + 1], c = in[3 * q + 2];
        // pixels: (a.x a.y a.z) (a.w b.x b.y) (b.z b.w c.x) (c.y c.z c.w)
        const uint32_t r0 = to_byte(a.x), g0 = to_byte(a.y), b0 = to_byte(a.z);
        const uint32_t r1 = to_byte(a.w), g1 = to_byte(b.x), b1 = to_byte(b.y);
        const uint32_t r2 = to_byte(b.z), g2 = to_byte(b.w), b2 = to_byte(c.x);
        const uint32_t r3 = to_byte(c.y), g3 = to_byte(c.z), b3 = to_byte(c.w);
        if constexpr (kLayout == XSG_IMG_HWC_RGB) {
            uint32_t* o = reinterpret_cast<uint32_t*>(out + 12 * q);
            o[0] = r0 | (g0 << 8) | (b0 << 16) | (r1 << 24);
            o[1] = g1 | (b1 << 8) | (r2 << 16) | (g2 << 24);
            o[2] = b2 | (r3 << 8) | (g3 << 16) | (b3 << 24);
        } else if constexpr (kLayout == XSG_IMG_HWC_RGBA) {
            reinterpret_cast<uint4*>(out)[q] =
                make_uint4(r0 | (g0 << 8) | (b0 << 16) | 0xff000000u, r1 | (g1 << 8) | (b1 << 16) | 0xff000000u,
                           r2 | (g2 << 8) | (b2 << 16) | 0xff000000u, r3 | (g3 << 8) | (b3 << 16) | 0xff000000u);
        } else {
            reinterpret_cast<uint32_t*>(out)[q] = r0 | (r1 << 8) | (r2 << 16) | (r3 << 24);
            reinterpret_cast<uint32_t*>(out + n_pixels)[q] = g0 | (g1 << 8) | (g2 << 16) | (g3 << 24);
            reinterpret_cast<uint32_t*>(out + 2 * n_pixels)[q] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
    }
}

// Pixels [first, n) one per thread.
template <int kLayout>
__global__ void __launch_bounds__(kImgThreads)
    image_bytes_kernel(const float* __restrict__ in, int64_t first, int64_t n, uint8_t* __restrict__ out) {
    const int64_t i = first + int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint8_t r = uint8_t(to_byte(in[3 * i])), g = uint8_t(to_byte(in[3 * i + 1])),
                  b = uint8_t(to_byte(in[3 * i + 2]));
    if constexpr (kLayout == XSG_IMG_HWC_RGB) {
        out[3 * i] = r; out[3 * i + 1] = g; out[3 * i + 2] = b;
    } else if constexpr (kLayout == XSG_IMG_HWC_RGBA) {
        out[4 * i] = r; out[4 * i + 1] = g; out[4 * i + 2] = b; out[4 * i + 3] = 255;
    } else {
        out[i] = r; out[n + i] = g; out[2 * n + i] = b;
    }
}

template <int kLayout>
void image_bytes(const float* in, int64_t n, uint8_t* out, cudaStream_t st) {
    const uintptr_t ia = reinterpret_cast<uintptr_t>(in), oa = reinterpret_cast<uintptr_t>(out);
    // vector stores: 16 B (RGBA), 4 B (RGB; CHW, whose planes start at
    // multiples of n, so n must be a multiple of 4 too)
    const bool vec = (ia % 16 == 0) && (kLayout == XSG_IMG_HWC_RGBA ? oa % 16 == 0 : oa % 4 == 0) &&
                     (kLayout != XSG_IMG_CHW_RGB || n % 4 == 0);
    int64_t done = 0;
    if (vec && n >= 4) {
        const int64_t quads = n / 4;
        const int64_t blocks = (quads + kImgThreads - 1) / kImgThreads;
        const unsigned grid = unsigned(blocks < 148 * 16 ? blocks : 148 * 16);
        launch(image_bytes_vec_kernel<kLayout>, grid, kImgThreads, 0, st, reinterpret_cast<const float4*>(in), quads,
               n, out);
        done = quads * 4;
    }
    if (done < n) launch(image_bytes_kernel<kLayout>, blocks_for(n - done, kImgThreads), kImgThreads, 0, st, in,
                         done, n, out);
}

}  // namespace xsg

using namespace xsg;

extern "C" int xsg_image_to_bytes(int layout, const float* image, int64_t n_pixels, uint8_t* out,
                                  xsg_stream_t stream) {
    XSG_REQUIRE(n_pixels >= 0, "image_to_bytes: negative pixel count");
    if (n_pixels == 0) return XSG_OK;
    XSG_REQUIRE(image && out, "image_to_bytes: null pointer");
    XSG_REQUIRE(reinterpret_cast<uintptr_t>(image) % 4 == 0, "image_to_bytes: image must be 4-byte aligned");
    switch (layout) {
        case XSG_IMG_HWC_RGB: image_bytes<XSG_IMG_HWC_RGB>(image, n_pixels, out, as_cuda(stream)); break;
        case XSG_IMG_HWC_RGBA: image_bytes<XSG_IMG_HWC_RGBA>(image, n_pixels, out, as_cuda(stream)); break;
        case XSG_IMG_CHW_RGB: image_bytes<XSG_IMG_CHW_RGB>(image, n_pixels, out, as_cuda(stream)); break;
        default: return set_error(XSG_ERR_INVALID_ARGUMENT, "image_to_bytes: unknown layout");
    }
    return check_launch("image_to_bytes");
}
