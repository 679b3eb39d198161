// Tensor-map (TMA descriptor) construction with a process-wide cache.
#include "gemm_host.h"

#include <cstring>
#include <mutex>

namespace qk {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Everything a descriptor is a function of.  Plain data: compared with memcmp, so it is zero-filled first.
struct MapKey {
  const void* base;
  unsigned long long dims[3];
  unsigned long long strides[2];
  unsigned int box[3];
  int rank, dtype, swizzle, l2promo;
};

// Direct-mapped: a slot is (key, descriptor); a collision overwrites.  512 slots x ~200 bytes.
constexpr int kSlots = 512;
struct Slot {
  bool used;
  MapKey key;
  CUtensorMap map;
};
Slot g_slots[kSlots];
std::mutex g_mu;
long long g_hits = 0, g_misses = 0;

unsigned long long hash_key(const MapKey& k) {
  const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
  unsigned long long h = 1469598103934665603ull;   // FNV-1a
  for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ p[i]) * 1099511628211ull;
  return h;
}

int encode_cached(CUtensorMap* tm, const MapKey& key, const char* what) {
  Slot& slot = g_slots[hash_key(key) % kSlots];
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (slot.used && memcmp(&slot.key, &key, sizeof(MapKey)) == 0) {
      *tm = slot.map;
      ++g_hits;
      return QK_OK;
    }
  }
  EncodeTiledFn enc = get_encode();
  if (!enc) return qk_fail(QK_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {key.dims[0], key.dims[1], key.dims[2]};
  cuuint64_t strides[2] = {key.strides[0], key.strides[1]};
  cuuint32_t box[3] = {key.box[0], key.box[1], key.box[2]};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = enc(tm, static_cast<CUtensorMapDataType>(key.dtype), static_cast<cuuint32_t>(key.rank),
                         const_cast<void*>(key.base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         static_cast<CUtensorMapSwizzle>(key.swizzle), static_cast<CUtensorMapL2promotion>(key.l2promo),
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return qk_fail(QK_ERR_CUDA, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", what, (int)r);
  std::lock_guard<std::mutex> lock(g_mu);
  slot.used = true;
  slot.key = key;
  slot.map = *tm;
  ++g_misses;
  return QK_OK;
}

}  // namespace

int make_operand_map(CUtensorMap* tm, const void* base, long long rows, long long kbytes, long long ld, int box_rows) {
  MapKey k;
  memset(&k, 0, sizeof(k));
  k.base = base;
  k.rank = 2;
  k.dims[0] = static_cast<unsigned long long>(kbytes);
  k.dims[1] = static_cast<unsigned long long>(rows);
  k.strides[0] = static_cast<unsigned long long>(ld);
  k.box[0] = 128u;
  k.box[1] = static_cast<unsigned int>(box_rows);
  k.dtype = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  k.swizzle = CU_TENSOR_MAP_SWIZZLE_128B;
  k.l2promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  return encode_cached(tm, k, "operand");
}

int make_scale_map(CUtensorMap* tm, const void* base, long long rm, long long rk, long long stride_rm, long long stride_rk,
                   int box_k, int box_mn) {
  MapKey k;
  memset(&k, 0, sizeof(k));
  k.base = base;
  k.rank = 3;
  k.dims[0] = 128u;
  k.dims[1] = static_cast<unsigned long long>(rk);
  k.dims[2] = static_cast<unsigned long long>(rm);
  k.strides[0] = static_cast<unsigned long long>(stride_rk);
  k.strides[1] = static_cast<unsigned long long>(stride_rm);
  k.box[0] = 128u;
  k.box[1] = static_cast<unsigned int>(box_k);
  k.box[2] = static_cast<unsigned int>(box_mn);
  k.dtype = CU_TENSOR_MAP_DATA_TYPE_UINT32;
  k.swizzle = CU_TENSOR_MAP_SWIZZLE_NONE;
  k.l2promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  return encode_cached(tm, k, "scales");
}

int make_store_map(CUtensorMap* tm, const void* base, int esize, long long rows, long long cols, long long ld_bytes,
                   int box_bytes) {
  MapKey k;
  memset(&k, 0, sizeof(k));
  k.base = base;
  k.rank = 2;
  k.dims[0] = static_cast<unsigned long long>(cols);
  k.dims[1] = static_cast<unsigned long long>(rows);
  k.strides[0] = static_cast<unsigned long long>(ld_bytes);
  k.box[0] = static_cast<unsigned int>(box_bytes / esize);
  k.box[1] = 32u;
  k.dtype = esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_UINT32 : esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  k.swizzle = box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
            : box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
            : box_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE;
  k.l2promo = CU_TENSOR_MAP_L2_PROMOTION_NONE;
  return encode_cached(tm, k, "output");
}

void tensor_map_cache_stats(long long* hits, long long* misses) {
  std::lock_guard<std::mutex> lock(g_mu);
  *hits = g_hits;
  *misses = g_misses;
}

}  // namespace qk

extern "C" void qk_tensor_map_cache_stats(long long* hits, long long* misses) { qk::tensor_map_cache_stats(hits, misses); }
