#include "tma_host.h"

#include <mutex>
#include <sstream>

namespace bdh {

namespace {
thread_local std::string g_last_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

int sm_count(int device) {
  static int cache[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[device] = n;
  }
  return cache[device];
}

bool make_map_4d(CUtensorMap* map, const void* base, int elem_bytes, const int64_t dims[4],
                 const int64_t strides_bytes[3], int box0, int box1, const char* what) {
  const int box[4] = {box0, box1, 1, 1};
  return make_map_4d_box(map, base, elem_bytes, dims, strides_bytes, box, what);
}

bool make_map_4d_box(CUtensorMap* map, const void* base, int elem_bytes, const int64_t dims[4],
                     const int64_t strides_bytes[3], const int box_in[4], const char* what) {
  const int box0 = box_in[0], box1 = box_in[1];
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the CUDA driver");
    return false;
  }
  // The driver call needs a current context. A thread that has not made a runtime call that
  // binds one yet (autograd's device thread, when the backward's first CUDA work is this
  // library) has none: bind the current device's primary context first.
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) {
    std::ostringstream os;
    os << what << ": base address must be 16-byte aligned for TMA";
    set_error(os.str());
    return false;
  }
  cuuint64_t gdim[4];
  cuuint64_t gstride[3];
  for (int i = 0; i < 4; ++i) gdim[i] = static_cast<cuuint64_t>(dims[i] > 0 ? dims[i] : 1);
  for (int i = 0; i < 3; ++i) {
    int64_t s = strides_bytes[i];
    // A size-1 dimension is never stepped; give it any legal stride.
    if (dims[i + 1] <= 1) s = 16;
    if (s <= 0 || (s % 16) != 0 || s >= (int64_t(1) << 40)) {
      std::ostringstream os;
      os << what << ": stride " << strides_bytes[i] << " B of dim " << (i + 1)
         << " is not a positive multiple of 16 B (TMA)";
      set_error(os.str());
      return false;
    }
    gstride[i] = static_cast<cuuint64_t>(s);
  }
  cuuint32_t box[4] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1),
                        static_cast<cuuint32_t>(box_in[2]), static_cast<cuuint32_t>(box_in[3])};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  CUtensorMapDataType dt =
      elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), gdim, gstride, box, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::ostringstream os;
    os << what << ": cuTensorMapEncodeTiled failed (CUresult " << static_cast<int>(r)
       << "), dims=[" << dims[0] << "," << dims[1] << "," << dims[2] << "," << dims[3]
       << "] strides_bytes=[" << strides_bytes[0] << "," << strides_bytes[1] << ","
       << strides_bytes[2] << "] box=[" << box0 << "," << box1 << "," << box_in[2] << ","
       << box_in[3] << "]";
    set_error(os.str());
    return false;
  }
  return true;
}

}  // namespace bdh
