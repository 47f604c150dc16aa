// common.cu — error reporting, device status word, tensor maps, ABI version.
#include "common.cuh"
#include "sm100.cuh"

#include <mutex>
#include <vector>

namespace sb {

static thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int num_sms() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> g(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int elem_bytes,
                 uint64_t rows, uint64_t cols, uint64_t row_stride_elems, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(SB_ERR_INVALID, "tensor base %p is not 16-byte aligned", base);
  if ((row_stride_elems * elem_bytes) % 16 != 0)
    return fail(SB_ERR_INVALID, "row stride of %llu bytes is not a multiple of 16",
                (unsigned long long)(row_stride_elems * elem_bytes));
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(SB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu box=%ux%u",
                (int)r, (unsigned long long)rows, (unsigned long long)cols, box_rows, box_cols);
  return SB_OK;
}

// ---------------------------------------------------------------------------
// per-kernel event profiler
// ---------------------------------------------------------------------------
namespace {
struct ProfEntry {
  std::string name;
  int64_t launches = 0;
  double total_ms = 0.0;
};
struct Pending {
  const char* name;
  cudaEvent_t start, stop;
};
std::mutex g_prof_mu;
bool g_prof_on = false;
std::vector<ProfEntry> g_prof_entries;
std::vector<Pending> g_prof_pending;
std::vector<cudaEvent_t> g_prof_free;

void prof_resolve_locked() {
  for (const Pending& p : g_prof_pending) {
    float ms = 0.f;
    if (cudaEventSynchronize(p.stop) == cudaSuccess &&
        cudaEventElapsedTime(&ms, p.start, p.stop) == cudaSuccess) {
      ProfEntry* e = nullptr;
      for (auto& x : g_prof_entries)
        if (x.name == p.name) e = &x;
      if (!e) {
        g_prof_entries.push_back(ProfEntry{p.name, 0, 0.0});
        e = &g_prof_entries.back();
      }
      e->launches += 1;
      e->total_ms += ms;
    }
    g_prof_free.push_back(p.start);
    g_prof_free.push_back(p.stop);
  }
  g_prof_pending.clear();
}
}  // namespace

bool prof_enabled() { return g_prof_on; }

cudaEvent_t prof_event() {
  std::lock_guard<std::mutex> g(g_prof_mu);
  if (!g_prof_free.empty()) {
    cudaEvent_t e = g_prof_free.back();
    g_prof_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

void prof_record(const char* name, cudaEvent_t start, cudaEvent_t stop) {
  std::lock_guard<std::mutex> g(g_prof_mu);
  g_prof_pending.push_back(Pending{name, start, stop});
  if (g_prof_pending.size() > 4096) prof_resolve_locked();
}

}  // namespace sb

extern "C" int sb_profile_enable(int on) {
  std::lock_guard<std::mutex> g(sb::g_prof_mu);
  sb::prof_resolve_locked();
  sb::g_prof_entries.clear();
  sb::g_prof_on = on != 0;
  return SB_OK;
}

extern "C" int sb_profile_count(void) {
  std::lock_guard<std::mutex> g(sb::g_prof_mu);
  sb::prof_resolve_locked();
  return (int)sb::g_prof_entries.size();
}

extern "C" int sb_profile_entry(int i, char* name, size_t len, int64_t* launches, double* total_ms) {
  std::lock_guard<std::mutex> g(sb::g_prof_mu);
  sb::prof_resolve_locked();
  if (i < 0 || i >= (int)sb::g_prof_entries.size())
    return sb::fail(SB_ERR_INVALID, "profile entry %d out of range", i);
  const auto& e = sb::g_prof_entries[i];
  if (name && len) {
    size_t n = e.name.size() < len - 1 ? e.name.size() : len - 1;
    memcpy(name, e.name.data(), n);
    name[n] = 0;
  }
  if (launches) *launches = e.launches;
  if (total_ms) *total_ms = e.total_ms;
  return SB_OK;
}

extern "C" int sb_abi_version(void) { return SB_ABI_VERSION; }

extern "C" int sb_last_error(char* buf, size_t len) {
  const std::string& s = sb::t_last_error;
  if (buf && len) {
    size_t n = s.size() < len - 1 ? s.size() : len - 1;
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return (int)s.size();
}

extern "C" int sb_device_status(int device) {
  int prev = 0;
  SB_CUDA_TRY(cudaGetDevice(&prev));
  SB_CUDA_TRY(cudaSetDevice(device));
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, sb::g_status, sizeof(v));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(sb::g_status, &zero, sizeof(zero));
  cudaSetDevice(prev);
  if (e != cudaSuccess)
    return sb::fail(SB_ERR_CUDA, "status read failed: %s", cudaGetErrorString(e));
  const unsigned waits = sb::ST_TIMEOUT_PRODUCER | sb::ST_TIMEOUT_MMA | sb::ST_TIMEOUT_EPILOGUE |
                         sb::ST_TIMEOUT_UNPACK | sb::ST_TIMEOUT_EP;
  if (v & waits)
    return sb::fail(SB_ERR_DEVICE_TIMEOUT, "device %d kernel status 0x%x (bounded wait expired)", device, v);
  if (v & sb::ST_RANGE)
    return sb::fail(SB_ERR_INVALID,
                    "device %d kernel status 0x%x (a non-finite value in a layer's output: a non-finite "
                    "input, or on the bf16 path a hidden value past fp16's 65504; fp32 inputs take the bf16 "
                    "hi/lo path, which has fp32's range)", device, v);
  if (v != 0)
    return sb::fail(SB_ERR_INVALID, "device %d kernel status 0x%x (an out-of-range expert id was dropped)",
                    device, v);
  return SB_OK;
}
