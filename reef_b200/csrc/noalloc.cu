// noalloc.cu -- reef_b200_linear_w8a8_noalloc: the W8A8 linear for callers
// that cannot allocate device memory at all, not even the quantisation
// scratch the other entry points ask the caller to provide.
//
// Some hosts own every byte of device memory through their own arena and
// forbid libraries from calling cudaMalloc (an inference engine with a fixed
// memory plan, or a port of reef's Coral firmware, whose kernels never
// allocate); others cannot afford the device-wide synchronisation a
// cudaMalloc may bring on a latency-critical path.  This entry point needs
// only the caller's inputs and outputs: its scratch (the int8 rows and their
// scales) is a fixed array in the library's own device image.
//
// The array is shared by every call on a device and keeps the last call's
// contents.  Calls that overlap on the GPU (two streams, or two host threads
// on one device) race on it and must be serialised by the caller.  Nothing in
// it has to start at zero: the quantiser writes every byte a call reads,
// including the row padding.
#include "../../include/reef_b200.h"

#include "ops.h"

#include <mutex>

namespace {

using namespace reef;

// The scratch: x_q [rows][kpad(in)] int8, then x_scale [rows] fp32 at the
// next 256-byte boundary.  Every GPU that loads the library holds these
// bytes until the process exits.
constexpr size_t kScratchBytes = static_cast<size_t>(REEF_B200_NOALLOC_SCRATCH_BYTES);
static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// The device address of g_scratch belongs to one CUDA context: the module that
// holds the array is loaded into each context separately, and a context that
// is destroyed (cudaDeviceReset, or a caller's own cuCtxDestroy) takes the
// array with it.  So the cache is keyed on the current context's unique id
// (cuCtxGetId, never reused within a process), not on the device index alone:
// a call made under a context the cache has not seen looks the address up
// again, with that context current.
using CtxGetCurrent = CUresult (*)(CUcontext*);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long*);

struct CtxFns {
  CtxGetCurrent current = nullptr;
  CtxGetId id = nullptr;
};

const CtxFns& ctx_fns() {
  static CtxFns fns;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fns.current = reinterpret_cast<CtxGetCurrent>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fns.id = reinterpret_cast<CtxGetId>(p);
  });
  return fns;
}

struct ScratchEntry {
  bool used = false;
  unsigned long long ctx_id = 0;
  void* ptr = nullptr;
};
constexpr int kMaxEntries = 64;
ScratchEntry g_scratch_dev[kMaxEntries];
int g_scratch_next = 0;  // round-robin victim once every entry is taken
std::mutex g_scratch_mu;

// The device address of g_scratch in the current context.  In host code the
// name g_scratch is only a stand-in for the symbol, never a device address,
// so it is looked up with the context current and cached under that
// context's id.
int scratch_ptr(void** out) {
  const CtxFns& f = ctx_fns();
  if (f.current == nullptr || f.id == nullptr) return kErrCuda;
  CUcontext ctx = nullptr;
  if (f.current(&ctx) != CUDA_SUCCESS) return kErrCuda;
  if (ctx == nullptr) {
    // no context is current on this thread yet: make the runtime's primary
    // context of the current device current (the one the kernels below
    // launch in); a context the caller made current is never replaced
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess ||
        f.current(&ctx) != CUDA_SUCCESS || ctx == nullptr)
      return kErrCuda;
  }
  unsigned long long id = 0;
  if (f.id(ctx, &id) != CUDA_SUCCESS) return kErrCuda;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  for (const ScratchEntry& e : g_scratch_dev)
    if (e.used && e.ctx_id == id) {
      *out = e.ptr;
      return kOk;
    }
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess || p == nullptr) return kErrCuda;
  int slot = -1;
  for (int i = 0; i < kMaxEntries; ++i)
    if (!g_scratch_dev[i].used) {
      slot = i;
      break;
    }
  if (slot < 0) slot = g_scratch_next++ % kMaxEntries;
  g_scratch_dev[slot] = ScratchEntry{true, id, p};
  *out = p;
  return kOk;
}

// Bytes of scratch a call uses: rows x kpad(in) int8, then rows fp32 scales.
size_t scratch_bytes(size_t rows, size_t in) {
  const size_t q = rows * kpad(in);
  return ((q + 255) / 256) * 256 + rows * sizeof(float);
}

}  // namespace

extern "C" int reef_b200_linear_w8a8_noalloc(size_t rows, size_t in, size_t out, const float* x,
                                             const int8_t* w, const float* w_scale,
                                             const float* bias, float* y,
                                             reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (in == 0 || out == 0 || rows > (1u << 31) - 1 || in > (1u << 31) - 1 ||
      out > (1u << 31) - 1 || !x || !w || !w_scale || !y)
    return REEF_B200_ERR_INVALID;
  if (scratch_bytes(rows, in) > kScratchBytes) return REEF_B200_ERR_TOO_LARGE;
  if (int rc = check_device()) return rc;
  void* base = nullptr;
  if (int rc = scratch_ptr(&base)) return rc;
  const long long ld = static_cast<long long>(kpad(in));
  int8_t* x_q = static_cast<int8_t*>(base);
  float* x_scale = reinterpret_cast<float*>(static_cast<unsigned char*>(base) +
                                            ((rows * kpad(in) + 255) / 256) * 256);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (int rc = quantize_rows(static_cast<long long>(rows), static_cast<long long>(in), x, x_q, ld,
                             x_scale, nullptr, st))
    return rc;
  GemmProblem p{};
  p.M = static_cast<int>(rows);
  p.N = static_cast<int>(out);
  p.K = static_cast<int>(in);
  p.a = x_q;
  p.lda = ld;
  p.b = w;
  p.ldb = ld;
  p.args.x_scale = x_scale;
  p.args.w_scale = w_scale;
  p.args.bias_f = bias;
  p.args.y = y;
  p.args.ldy = static_cast<long long>(out);
  return gemm_i8(p, kEpiF32W8A8, st);
}
