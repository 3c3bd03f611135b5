// Host video crop -> device buffer as one strided DMA (render_tiled's tile loader).
//
// The reference crops a CPU video with a strided view and `.to(dev, non_blocking=True)`
// (tiling.py:190), which packs the view into a contiguous host copy first.  When the host
// video is pinned, the copy engine can read the crop's rows straight from it: the video is
// `planes` planes of `src_rows` rows with a pitch of `src_pitch` bytes, and the crop is the
// window of `height` rows of `width_bytes` bytes starting at byte `x_bytes` of row `y` in
// every plane, written densely ([planes, height, width_bytes]) to dst.  No host thread
// touches the pixels, so ranks that share a host do not contend for its memory bandwidth.
#include "common.cuh"

extern "C" {

int fvb_copy_window_h2d(const void* src, int64_t src_pitch, int64_t src_rows, int64_t planes,
                        int64_t x_bytes, int64_t y, int64_t width_bytes, int64_t height,
                        void* dst, fvb_stream_t stream) {
  using namespace fvb;
  FVB_REQUIRE(src && dst, "fvb_copy_window_h2d: NULL pointer");
  FVB_REQUIRE(src_pitch > 0 && src_rows > 0 && planes >= 0 && x_bytes >= 0 && y >= 0 &&
                  width_bytes >= 0 && height >= 0,
              "fvb_copy_window_h2d: negative or zero size");
  FVB_REQUIRE(x_bytes + width_bytes <= src_pitch && y + height <= src_rows,
              "fvb_copy_window_h2d: window [%lld, %lld) x [%lld, %lld) outside the %lld x %lld "
              "byte plane", (long long)x_bytes, (long long)(x_bytes + width_bytes), (long long)y,
              (long long)(y + height), (long long)src_pitch, (long long)src_rows);
  if (planes == 0 || width_bytes == 0 || height == 0) return FVB_OK;
  cudaMemcpy3DParms p = {};
  p.srcPtr = make_cudaPitchedPtr(const_cast<void*>(src), (size_t)src_pitch, (size_t)src_pitch,
                                 (size_t)src_rows);
  p.srcPos = make_cudaPos((size_t)x_bytes, (size_t)y, 0);
  p.dstPtr = make_cudaPitchedPtr(dst, (size_t)width_bytes, (size_t)width_bytes, (size_t)height);
  p.dstPos = make_cudaPos(0, 0, 0);
  p.extent = make_cudaExtent((size_t)width_bytes, (size_t)height, (size_t)planes);
  p.kind = cudaMemcpyHostToDevice;
  FVB_CUDA_TRY(cudaMemcpy3DAsync(&p, (cudaStream_t)stream), "fvb_copy_window_h2d");
  return FVB_OK;
}

}  // extern "C"
