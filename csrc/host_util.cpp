#include "host_util.h"

#include <cstdlib>
#include <mutex>
#include <vector>

namespace pb {

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    PB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    PB_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr,
             "cuTensorMapEncodeTiled entry point not found");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

std::mutex g_err_mu;
std::vector<int*> g_err_words;
std::vector<unsigned> g_split_next;

// Device block per GPU: the 256-byte error word area, then kSplitSlots
// counter slots of kSplitSlotInts ints for the ordered split-K epilogue.
constexpr size_t kErrBytes = 256;
constexpr size_t kBlockBytes = kErrBytes + (size_t)kSplitSlots * kSplitSlotInts * sizeof(int);

int cur_device(int device) {
  if (device >= 0) return device;
  int d = 0;
  PB_CUDA_CHECK(cudaGetDevice(&d));
  return d;
}
}  // namespace

bool pdl_enabled() {
  // off unless PB_PDL=1: measured on B200 at the Qwen3-0.6B step (CUDA-graph
  // replays), the step time did not change (46.4-46.5 ms either way)
  static const bool on = [] {
    const char* v = getenv("PB_PDL");
    return v && v[0] == '1';
  }();
  return on;
}

int* error_word(int device) {
  device = cur_device(device);
  std::lock_guard<std::mutex> lk(g_err_mu);
  if ((int)g_err_words.size() <= device) g_err_words.resize(device + 1, nullptr);
  if (!g_err_words[device]) {
    int prev = 0;
    PB_CUDA_CHECK(cudaGetDevice(&prev));
    PB_CUDA_CHECK(cudaSetDevice(device));
    int* p = nullptr;
    PB_CUDA_CHECK(cudaMalloc(&p, kBlockBytes));
    PB_CUDA_CHECK(cudaMemset(p, 0, kBlockBytes));
    PB_CUDA_CHECK(cudaSetDevice(prev));
    g_err_words[device] = p;
  }
  return g_err_words[device];
}

int* split_counters(int device) {
  device = cur_device(device);
  int* base = error_word(device);
  std::lock_guard<std::mutex> lk(g_err_mu);
  if ((int)g_split_next.size() <= device) g_split_next.resize(device + 1, 0u);
  const unsigned slot = g_split_next[device]++ % kSplitSlots;
  return base + kErrBytes / sizeof(int) + (size_t)slot * kSplitSlotInts;
}

int read_error(int device) {
  int v = 0;
  PB_CUDA_CHECK(cudaMemcpy(&v, error_word(device), sizeof(int), cudaMemcpyDeviceToHost));
  return v;
}

void clear_error(int device) {
  // a kernel that gave up may have left split-K counters mid-count: reset them too
  PB_CUDA_CHECK(cudaMemset(error_word(device), 0, kBlockBytes));
}

int num_sms(int device) {
  static int cache[64] = {0};
  device = cur_device(device);
  if (device < 64 && cache[device]) return cache[device];
  int n = 0;
  PB_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  if (device < 64) cache[device] = n;
  return n;
}

CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer,
                              uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer,
                              bool swizzle128) {
  PB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  PB_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (2d) failed: code " + std::to_string(r));
  return m;
}

CUtensorMap make_tmap_2d_bf16_swz(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                                  uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  PB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  PB_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  else if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  else if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  else PB_CHECK(swizzle_bytes == 0, "TMA swizzle must be 0, 32, 64 or 128 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (2d, swizzled store) failed: code " + std::to_string(r));
  return m;
}

CUtensorMap make_tmap_3d_bf16(const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                              uint64_t stride1_elems, uint64_t stride2_elems, uint32_t b0,
                              uint32_t b1, uint32_t b2) {
  PB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  PB_CHECK((stride1_elems * 2) % 16 == 0 && (stride2_elems * 2) % 16 == 0,
           "TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_elems * 2, stride2_elems * 2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3d) failed: code " + std::to_string(r));
  return m;
}

CUtensorMap make_tmap_3d_f32(void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_elems,
                             uint64_t stride2_elems, uint32_t b0, uint32_t b1, uint32_t b2, bool swizzle128) {
  PB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  PB_CHECK((stride1_elems * 4) % 16 == 0 && (stride2_elems * 4) % 16 == 0,
           "TMA strides must be multiples of 16 bytes");
  PB_CHECK(!swizzle128 || b0 * 4 <= 128, "128B swizzle needs an inner box of at most 128 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_elems * 4, stride2_elems * 4};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  PB_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3d f32) failed: code " + std::to_string(r));
  return m;
}

}  // namespace pb
