// libjeffb200: one translation unit (no relocatable device code), host utilities of the C ABI.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "common.cuh"

namespace jb {

__device__ int g_device_status;   // set by kernels whose bounded waits gave up (JB_DEV_TIMEOUT | where)

static thread_local char g_error[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

int status_of(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return JB_OK;
  set_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return JB_ECUDA;
}

int check_launch(const char* what) { return status_of(cudaGetLastError(), what); }

int* device_status_word() {
  static std::mutex mu;
  static int* addr[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    addr[dev] = static_cast<int*>(p);
  }
  return addr[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool pdl_enabled() {
  static const bool on = getenv("JB_NO_PDL") == nullptr;
  return on;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t outer,
                 uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return JB_ECUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15)) {
    set_error("tensor map: base %p and row pitch %llu must be 16-byte aligned", base, (unsigned long long)row_bytes);
    return JB_EINVAL;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d): dims %llu x %llu, pitch %llu, box %u x %u", (int)r,
              (unsigned long long)inner, (unsigned long long)outer, (unsigned long long)row_bytes, box_inner,
              box_outer);
    return JB_ECUDA;
  }
  return JB_OK;
}

int make_tmap_planes(CUtensorMap* map, const void* base, uint64_t rows, uint32_t cols, uint64_t row_bytes,
                     uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return JB_ECUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15) || cols % 8 || cols == 0 || cols > 64) {
    set_error("planes map: base %p, row pitch %llu, %u columns (16-byte aligned, columns a multiple of 8 up to 64)",
              base, (unsigned long long)row_bytes, cols);
    return JB_EINVAL;
  }
  cuuint64_t dims[3] = {8, rows, cols / 8};
  cuuint64_t strides[2] = {row_bytes, 16};
  cuuint32_t box[3] = {8, box_rows, cols / 8};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled (planes) failed (%d): %llu rows x %u columns, pitch %llu", (int)r,
              (unsigned long long)rows, cols, (unsigned long long)row_bytes);
    return JB_ECUDA;
  }
  return JB_OK;
}

int make_tmap_nd(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int rank, const uint64_t* dims,
                 const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return JB_ECUDA;
  }
  if (rank < 1 || rank > 5 || (reinterpret_cast<uintptr_t>(base) & 15)) {
    set_error("tensor map: rank %d, base %p (16-byte aligned, rank 1..5)", rank, base);
    return JB_EINVAL;
  }
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], elem[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    elem[i] = 1;
    if (i + 1 < rank) {
      st[i] = strides[i];
      if (strides[i] & 15) {
        set_error("tensor map: stride %d of %llu bytes is not a multiple of 16", i, (unsigned long long)strides[i]);
        return JB_EINVAL;
      }
    }
  }
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for a rank-%d map", (int)r, rank);
    return JB_ECUDA;
  }
  return JB_OK;
}

}  // namespace jb

#include "lora_shrink_tc.cu"
#include "w4a16_gemm.cu"
#include "elementwise.cu"
#include "gdn.cu"
#include "gdn_chunk.cu"
#include "gdn_tc.cu"
#include "attention.cu"
#include "attention_tc.cu"

extern "C" int jb_abi_version(void) { return 2; }

extern "C" const char* jb_last_error(void) { return jb::g_error; }

extern "C" int jb_device_status(int* status, int reset, void* stream) {
  JB_REQUIRE(status, "jb_device_status: null status");
  int* word = jb::device_status_word();
  if (!word) {
    jb::set_error("jb_device_status: no device status word on this device");
    return JB_ECUDA;
  }
  cudaStream_t st = (cudaStream_t)stream;
  int r = jb::status_of(cudaMemcpyAsync(status, word, sizeof(int), cudaMemcpyDeviceToHost, st), "status read");
  if (r) return r;
  if (reset) {
    r = jb::status_of(cudaMemsetAsync(word, 0, sizeof(int), st), "status reset");
    if (r) return r;
  }
  return jb::status_of(cudaStreamSynchronize(st), "status sync");
}
