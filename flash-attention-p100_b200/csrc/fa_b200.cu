// fa_b200.cu -- the C ABI (include/fa_b200.h): argument checks, TMA tensor
// maps, kernel launches on the caller's stream, and the device error word.
//
// Host-side counterpart of the reference's torch binding
// (fa_p100_ext.cu:31-147): the same validation (fa_p100_ext.cu:55-65,
// :106-115) reported as status codes instead of TORCH_CHECK, the same
// scale = 1/sqrt(D) (:71, :117) and GROUP = Hq / Hkv (:66), but no allocation
// (the caller owns every buffer) and an explicit stream instead of the legacy
// default stream (flash_fwd.cuh:350).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <queue>
#include <vector>

#include "../../include/fa_b200.h"
#include "fa_bwd.cuh"
#include "fa_fwd.cuh"
#include "fa_fwd_persist.cuh"

namespace fab {

// Device error word: set by a kernel whose bounded wait gave up.
__device__ int g_device_error;

// Scratch for fa_b200_backward_noalloc: the backward's per-row workspace (Dv
// and LSE*log2e, two floats per padded query row, B*Hq*roundup(N,128) rows)
// lives here instead of in caller-provided memory. It is a fixed 16 MiB on every
// GPU that loads this library, for as long as the process lives. Host code
// cannot use the symbol's name as a device address; the address is fetched
// once per device with cudaGetSymbolAddress.
constexpr size_t kNoAllocRows = size_t(1) << 21;  // 2,097,152 padded rows x 8 B = 16 MiB
static __device__ __align__(256) float g_noalloc_scratch[2 * kNoAllocRows];

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int status = FA_B200_OK;
  int* err = nullptr;  // address of g_device_error on this device
  int sms = 148;       // multiprocessors
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
float* g_noalloc_ptr[kMaxDevices] = {};  // device address of g_noalloc_scratch
EncodeTiledFn g_encode = nullptr;

// Detail of the most recent failure on this host thread (fa_b200_last_error).
thread_local char g_last_error[512] = "";

void set_last_error(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

template <typename K>
void set_smem(K kernel, int bytes) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Opt every kernel of one element type (fp16, or bf16 when BF) in to its
// dynamic shared memory.
template <bool BF>
void set_smem_all() {
  set_smem(fwd_kernel_s<64, BF>, FwdCfgS<64>::SMEM);
  set_smem(fwd_kernel_s<128, BF>, FwdCfgS<128>::SMEM);
  set_smem(fwd_kernel_p<64, BF>, FwdCfgP<64>::SMEM);
  set_smem(fwd_kernel_p<128, BF>, FwdCfgP<128>::SMEM);
  set_smem(bwd_dkdv_kernel<64, BF>, DkdvCfg<64>::SMEM);
  set_smem(bwd_dkdv_kernel<128, BF>, DkdvCfg<128>::SMEM);
  set_smem(bwd_dq_kernel<64, BF>, DqCfg<64>::SMEM);
  set_smem(bwd_dq_kernel<128, BF>, DqCfg<128>::SMEM);
  set_smem(bwd_fused_kernel<64, BF>, FusedCfg<64>::SMEM);
  set_smem(bwd_fused_kernel<128, BF>, FusedCfg<128>::SMEM);
}

// One-time, per-device set-up with that device current: architecture check,
// opt-in to large dynamic shared memory, and the error word's address.
int device_setup(int* dev_out, int** err_out, int* sms_out = nullptr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return FA_B200_ERR_DEVICE;
  // Bind the device's primary context to this host thread. The tensor-map
  // encoder is a driver call and needs a current context; a caller's worker
  // thread (torch's autograd thread, for one) may not have one yet.
  if (cudaSetDevice(dev) != cudaSuccess) return FA_B200_ERR_DEVICE;
  *dev_out = dev;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& st = g_dev[dev];
  if (!st.ready) {
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev);
    if (major != 10) {
      st.status = FA_B200_ERR_DEVICE;
    } else {
      if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault,
                                             &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
          g_encode = reinterpret_cast<EncodeTiledFn>(fn);
      }
      void* addr = nullptr;
      if (!g_encode || cudaGetSymbolAddress(&addr, g_device_error) != cudaSuccess) {
        st.status = FA_B200_ERR_DEVICE;
      } else {
        st.err = static_cast<int*>(addr);
        set_smem_all<false>();
        set_smem_all<true>();
        st.status = (cudaGetLastError() == cudaSuccess) ? FA_B200_OK : FA_B200_ERR_DEVICE;
      }
    }
    st.ready = true;
  }
  *err_out = st.err;
  if (sms_out) *sms_out = st.sms;
  return st.status;
}

// 3-D fp16 (or fp32) tensor (slices, rows, cols) with 128-byte swizzled boxes
// of box_rows x (128 bytes of columns). Rows past `rows` read as zero.
bool make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes,
              uint64_t cols, uint64_t rows, uint64_t slices, uint32_t box_rows) {
  const cuuint64_t dims[3] = {cols, rows, slices};
  const cuuint64_t strides[2] = {cols * elem_bytes, cols * rows * elem_bytes};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / elem_bytes), box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    set_last_error(
        "cuTensorMapEncodeTiled -> CUresult %d for base %p (map at %p), dims {%llu, %llu, %llu}, "
        "strides {%llu, %llu} bytes, box {%u, %u, 1}",
        static_cast<int>(r), base, static_cast<void*>(m), static_cast<unsigned long long>(cols),
        static_cast<unsigned long long>(rows), static_cast<unsigned long long>(slices),
        static_cast<unsigned long long>(strides[0]), static_cast<unsigned long long>(strides[1]),
        box[0], box[1]);
  return r == CUDA_SUCCESS;
}

// 4-D view (D, N, H, B) of a (B, H, N, D) tensor with element strides `st`
// (the D axis contiguous), 128-byte swizzled boxes of box_rows x 128 bytes of
// columns. Rows past N read as zero; reduce-adds skip them.
bool make_map4(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes,
               uint64_t cols, uint64_t rows, uint64_t heads, uint64_t batch, const Strides& st,
               uint32_t box_rows) {
  const cuuint64_t dims[4] = {cols, rows, heads, batch};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(st.n) * elem_bytes,
                                 static_cast<cuuint64_t>(st.h) * elem_bytes,
                                 static_cast<cuuint64_t>(st.b) * elem_bytes};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / elem_bytes), box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = g_encode(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    set_last_error(
        "cuTensorMapEncodeTiled -> CUresult %d for base %p, dims {%llu, %llu, %llu, %llu}, "
        "strides {%llu, %llu, %llu} bytes, box {%u, %u, 1, 1}",
        static_cast<int>(r), base, static_cast<unsigned long long>(cols),
        static_cast<unsigned long long>(rows), static_cast<unsigned long long>(heads),
        static_cast<unsigned long long>(batch), static_cast<unsigned long long>(strides[0]),
        static_cast<unsigned long long>(strides[1]), static_cast<unsigned long long>(strides[2]),
        box[0], box[1]);
  return r == CUDA_SUCCESS;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

Strides contiguous(int H, int N, int D) {
  return Strides{static_cast<long long>(H) * N * D, static_cast<long long>(N) * D, D};
}

// Element strides a tensor map and 16-byte vector accesses can use: every
// stride non-negative and a multiple of 16 bytes.
bool strides_ok(const Strides& st, int elem_bytes) {
  const long long unit = 16 / elem_bytes;
  return st.b >= 0 && st.h >= 0 && st.n >= 0 && st.b % unit == 0 && st.h % unit == 0 &&
         st.n % unit == 0;
}

struct FwdLayout { Strides q, k, v, o; };
struct BwdLayout { Strides q, k, v, dO, o, dq, dk, dv; };

// FA_B200_OK, or FA_B200_ERR_LAUNCH with the CUDA error of the launch just made
// (and its kernel's name) as the thread's last-error detail.
int launch_status(const char* kernel) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return FA_B200_OK;
  set_last_error("launch of %s failed: %s", kernel, cudaGetErrorString(e));
  return FA_B200_ERR_LAUNCH;
}

// An fp32 dQ is produced by the fused kernel: one pass, dQ added into the
// zeroed output by TMA reduce-adds (the reference's fp32 dQ contract, and like
// its atomicAdd not bitwise deterministic). An fp16 dQ has no fp32 buffer to
// add into and takes the separate dK/dV and dQ kernels, which own every output
// row outright and are bitwise deterministic.
int default_stages(int dq_fp32) {
  return dq_fp32 ? (FA_B200_STAGE_ROWSUM | FA_B200_STAGE_FUSED) : FA_B200_STAGE_ALL;
}

// Device address of g_noalloc_scratch on `dev`, looked up once per device with
// that device current (device_setup has just made it current on this thread).
float* noalloc_scratch(int dev) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_noalloc_ptr[dev]) {
    float* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) {
      set_last_error("cudaGetSymbolAddress(g_noalloc_scratch) failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    g_noalloc_ptr[dev] = ptr;
  }
  return g_noalloc_ptr[dev];
}

// Longest sequence: padded row counts (N rounded up to 128) and per-row
// offsets stay well inside a 32-bit int.
constexpr int kMaxN = 1 << 30;

int check_shape(int B, int Hq, int Hkv, int N, int D) {
  if (D != 64 && D != 128) return FA_B200_ERR_HEAD_DIM;
  if (B < 1 || N < 1 || Hkv < 1 || Hq < 1 || Hq % Hkv != 0) return FA_B200_ERR_SHAPE;
  if (N > kMaxN) return FA_B200_ERR_TOO_LARGE;
  return FA_B200_OK;
}

// Fused backward CTA order: the (batch, kv-head) slices are taken in groups of
// head_group, and inside a group causal key block 0 of every slice comes first,
// then block 1, and so on; the GPU hands CTAs to SMs in that order as they free
// up. Small groups keep the CTAs that run together on few slices, so their
// Q/dO tiles and fp32 dQ rows stay in L2; but the last group's long causal
// CTAs then start late and finish alone. fused_makespan replays that dispatch
// (greedy, one CTA per SM) in units of query steps, a CTA costing
// kFusedCtaFixed steps (measured: 5.5 us against 3.15 us a step at D = 128)
// plus its own; fused_plan weighs each candidate's makespan by an L2 penalty measured on B200 (the same workload took 2.7%,
// 4.6% and 9.2% longer per step with 1.6x, 3.2x and 6.4x the footprint of a
// 64 MiB group at B=4, Hq=32, Hkv=8, N=3000): 3.5% per doubling past 64 MiB.
constexpr double kFusedCtaFixed = 1.7;
constexpr double kFusedReduceEpilogue = 0.3;   // fp32 dK/dV reduce-adds instead of 16-bit stores
constexpr uint64_t kFusedGroupBytes = 64ull << 20;

double fused_makespan(uint64_t bhkv, int nkb, int gsplit, int gper, int group, bool causal,
                      uint64_t hg, int sms, double fixed) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int s = 0; s < sms; ++s) free_at.push(0.0);
  double end = 0.0;
  for (uint64_t g0 = 0; g0 < bhkv; g0 += hg) {
    const uint64_t slices = std::min(hg, bhkv - g0);
    for (int kvb = 0; kvb < nkb; ++kvb) {
      const int qsteps = causal ? nkb - kvb : nkb;
      for (uint64_t s = 0; s < slices; ++s)
        for (int sp = 0; sp < gsplit; ++sp) {
          const int heads = std::min(gper, group - sp * gper);
          const double t = free_at.top() + fixed + static_cast<double>(heads) * qsteps;
          free_at.pop();
          free_at.push(t);
          end = std::max(end, t);
        }
    }
  }
  return end;
}

// Slices per scheduling group for the fused backward and the plan's cost
// (replayed makespan x L2 penalty, in query steps; 0 when the grid is too
// large to need a replay); cached per shape, since the replay costs up to a
// few milliseconds of host time.
struct FusedPlan {
  int hg;
  double cost;
};

FusedPlan fused_plan(uint64_t bhkv, int nkb, int gsplit, int gper, int group, bool causal, int N,
                     int D, int sms, bool reduce_epilogue) {
  // a slice's fp32 dQ rows and 16-bit Q/dO tiles: group * N * D * 8 bytes
  const uint64_t slice_bytes = std::max<uint64_t>(static_cast<uint64_t>(group) * N * D * 8, 1);
  const uint64_t hg_max = std::max<uint64_t>(1, kFusedGroupBytes / slice_bytes);
  const uint64_t n_l2 = (bhkv + hg_max - 1) / hg_max;
  const uint64_t hg_l2 = (bhkv + n_l2 - 1) / n_l2;     // equal groups within the L2 budget
  // Past 32 waves of CTAs a late start costs the makespan under 2%: the
  // L2-sized groups stand, without a replay.
  const uint64_t ctas = bhkv * static_cast<uint64_t>(nkb) * gsplit;
  if (ctas > 32ull * static_cast<uint64_t>(sms)) return {static_cast<int>(hg_l2), 0.0};
  const double fixed = kFusedCtaFixed + (reduce_epilogue ? kFusedReduceEpilogue : 0.0);
  using Key = std::array<long long, 9>;
  static std::mutex mu;
  static std::map<Key, FusedPlan> cache;
  const Key key{static_cast<long long>(bhkv), nkb, gsplit, gper, group, causal ? 1 : 0,
                static_cast<long long>(slice_bytes), sms, reduce_epilogue ? 1 : 0};
  {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  FusedPlan best{static_cast<int>(hg_l2), 1e300};
  uint64_t last = 0;
  for (uint64_t ng = n_l2; ng >= 1; --ng) {
    const uint64_t hg = (bhkv + ng - 1) / ng;
    if (hg == last) continue;
    last = hg;
    const double over = static_cast<double>(hg * slice_bytes) / static_cast<double>(kFusedGroupBytes);
    if (ng < n_l2 && over > 8.0) break;   // a penalty above 10%: larger groups cannot win
    const double cost = fused_makespan(bhkv, nkb, gsplit, gper, group, causal, hg, sms, fixed) *
                        (1.0 + 0.035 * std::max(0.0, std::log2(over)));
    if (cost < best.cost) best = {static_cast<int>(hg), cost};
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() >= 4096) cache.clear();   // bounded for callers that sweep many shapes
  cache.emplace(key, best);
  return best;
}

// The fused backward's schedule: a GQA group may be split over gsplit CTAs of
// gper heads each, which add their partial dK/dV into an fp32 accumulator (the
// caller's dk/dv when accumulating, else workspace when the caller sized it
// with fa_b200_backward_workspace_bytes_gqa: can_split); head_group slices are
// scheduled together.
struct FusedChoice {
  int gsplit, gper, head_group;
};

FusedChoice choose_fused(uint64_t bhkv, int nkb, int group, bool causal, int N, int D, int sms,
                         bool accumulate, bool can_split) {
  FusedChoice c{1, group, 1};
  const uint64_t units = bhkv * static_cast<uint64_t>(nkb);
  if (group > 1 && can_split && units < 2ull * sms) {
    // Too few (batch, kv-head) x key-block CTAs to fill the GPU. Heads per
    // CTA: the fewest waves of CTAs times the work of each (gper heads plus a
    // quarter head of fixed cost per CTA); more parts mean more fp32 dK/dV
    // partials to add, which are small at these sizes.
    double best = 1e30;
    for (int gp = 1; gp <= group; ++gp) {
      const uint64_t parts = (group + gp - 1) / gp;
      const uint64_t waves = (units * parts + sms - 1) / sms;
      const double cost = static_cast<double>(waves) * (gp + 0.25);
      if (cost < best) {
        best = cost;
        c.gper = gp;
      }
    }
    c.gsplit = (group + c.gper - 1) / c.gper;
    c.head_group = fused_plan(bhkv, nkb, c.gsplit, c.gper, group, causal, N, D, sms, true).hg;
  } else if (group > 1 && can_split) {
    // A grid that fills the GPU: split the group only when the replayed
    // makespan, with the split's accumulator memset and conversion pass
    // (HBM-bound, ~6 TB/s; none when the caller accumulates into fp32 dK/dV
    // already) counted in query steps, comes out at least 3% shorter --
    // typically equal-length non-causal CTAs that leave a last wave mostly
    // empty, such as the 8192-row pieces of an 8-way ring.
    const double acc_bytes = 8.0 * static_cast<double>(bhkv) * N * D;
    const double step_us = (D == 128) ? 3.15 : 1.8;
    const double extra = accumulate ? 0.0 : (5.0 + 2.5 * acc_bytes / 6.0e6) / step_us;
    FusedPlan best = fused_plan(bhkv, nkb, 1, group, group, causal, N, D, sms, accumulate);
    c.head_group = best.hg;
    for (int parts = 2; parts <= group && best.cost > 0.0; ++parts) {
      if (group % parts != 0) continue;
      const FusedPlan s = fused_plan(bhkv, nkb, parts, group / parts, group, causal, N, D, sms, true);
      if (s.cost > 0.0 && (s.cost + extra) < 0.97 * best.cost) {
        best = {s.hg, s.cost + extra};
        c = {parts, group / parts, s.hg};
      }
    }
  } else {
    c.head_group = fused_plan(bhkv, nkb, 1, group, group, causal, N, D, sms, accumulate).hg;
  }
  return c;
}

// The two-tile forward (256 query rows per CTA) when its grid fills the GPU,
// else the small-grid one (128 rows per CTA, 256-key steps).
bool forward_small_grid(int B, int Hq, int N, int sms) {
  return static_cast<long long>(B) * Hq * ((N + 255) / 256) < sms;
}

template <int D, bool BF>
int launch_forward(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                   int Hkv, int N, int causal, const FwdLayout& L, int sms, cudaStream_t stream,
                   int* err) {
  CUtensorMap tq, tk, tv;
  const uint64_t BH = static_cast<uint64_t>(B) * Hq;
  const CUtensorMapDataType dt = BF ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (!make_map4(&tq, q, dt, 2, D, N, Hq, B, L.q, 128) ||
      !make_map4(&tk, k, dt, 2, D, N, Hkv, B, L.k, 128) ||
      !make_map4(&tv, v, dt, 2, D, N, Hkv, B, L.v, 128))
    return FA_B200_ERR_TENSOR_MAP;
  FwdParams p = {};
  p.o = static_cast<uint16_t*>(o);
  p.so = L.o;
  p.lse = lse;
  p.err = err;
  p.n = N;
  p.hq = Hq;
  p.group = Hq / Hkv;
  p.causal = causal ? 1 : 0;
  p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)) * 1.4426950408889634);
  if (BH > 0x7fffffffull) return FA_B200_ERR_TOO_LARGE;
  CUtensorMap to;   // O output, 64-column x 128-row boxes
  if (!make_map4(&to, o, dt, 2, D, N, Hq, B, L.o, 128)) return FA_B200_ERR_TENSOR_MAP;
  if (forward_small_grid(B, Hq, N, sms)) {
    p.n_mblocks = (N + 127) / 128;
    if (p.n_mblocks > 65535) return FA_B200_ERR_TOO_LARGE;
    fwd_kernel_s<D, BF><<<dim3(static_cast<unsigned>(BH), p.n_mblocks), FwdCfgS<D>::THREADS,
                          FwdCfgS<D>::SMEM, stream>>>(tq, tk, tv, to, p);
    return launch_status("fwd_kernel_s");
  }
  p.n_mblocks = (N + 255) / 256;
  if (p.n_mblocks > 65535) return FA_B200_ERR_TOO_LARGE;
  // persistent: one CTA per SM walks the (batch, head, m-block) items
  const long long items = static_cast<long long>(BH) * p.n_mblocks;
  if (items > 0x7fffffffLL) return FA_B200_ERR_TOO_LARGE;
  p.n_items = static_cast<int>(items);
  p.bh_count = static_cast<int>(BH);
  const int grid = static_cast<int>(std::min<long long>(items, sms));
  fwd_kernel_p<D, BF><<<grid, FwdCfgP<D>::THREADS, FwdCfgP<D>::SMEM, stream>>>(tq, tk, tv, to, p);
  return launch_status("fwd_kernel_p");
}

template <int D, bool BF>
int launch_backward(const void* q, const void* k, const void* v, const void* dO, const void* o,
                    const float* lse, void* dq, int dq_fp32, void* dk, void* dv, float* ws,
                    size_t ws_bytes, int B, int Hq, int Hkv, int N, int causal, int stages,
                    const BwdLayout& L, int sms, cudaStream_t stream, int* err) {
  const uint64_t BH = static_cast<uint64_t>(B) * Hq, BHkv = static_cast<uint64_t>(B) * Hkv;
  const int nq128 = (N + 127) / 128;
  if (nq128 > 65535 || BH > 0x7fffffffull) return FA_B200_ERR_TOO_LARGE;
  // Every operand tile of the gradient kernels is 128 rows.
  CUtensorMap tq, tdo, tk, tv;
  const CUtensorMapDataType dt = BF ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (!make_map4(&tq, q, dt, 2, D, N, Hq, B, L.q, 128) ||
      !make_map4(&tdo, dO, dt, 2, D, N, Hq, B, L.dO, 128) ||
      !make_map4(&tk, k, dt, 2, D, N, Hkv, B, L.k, 128) ||
      !make_map4(&tv, v, dt, 2, D, N, Hkv, B, L.v, 128))
    return FA_B200_ERR_TENSOR_MAP;
  BwdParams p;
  p.o = static_cast<const uint16_t*>(o);
  p.dO = static_cast<const uint16_t*>(dO);
  p.so = L.o;
  p.sdo = L.dO;
  p.sdq = L.dq;
  p.sdk = L.dk;
  p.sdv = L.dv;
  p.lse = lse;
  const int n_pad = pad_rows(N);
  const long long rows_pad = static_cast<long long>(BH) * n_pad;
  p.dvec = ws;
  p.lse2 = ws + rows_pad;
  p.n_pad = n_pad;
  p.dq = dq;
  p.dk = static_cast<uint16_t*>(dk);
  p.dv = static_cast<uint16_t*>(dv);
  p.err = err;
  p.n = N;
  p.hq = Hq;
  p.group = Hq / Hkv;
  p.causal = causal ? 1 : 0;
  p.dq_fp32 = dq_fp32 ? 1 : 0;
  p.head_group = 1;
  p.gsplit = 1;
  p.gper = p.group;
  p.n_batch = B;
  p.dkv_acc = nullptr;
  // FA_B200_STAGE_ACCUMULATE: dq is added into (not zeroed), dk/dv are fp32
  // accumulators the fused kernel adds into
  const bool accumulate = (stages & FA_B200_STAGE_ACCUMULATE) != 0;
  p.dkv_reduce = accumulate ? 1 : 0;
  p.scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
  p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)) * 1.4426950408889634);

  if (stages & FA_B200_STAGE_ROWSUM) {
    const long long threads = rows_pad * (D / 8);
    bwd_preprocess_kernel<D, BF><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
        static_cast<const uint16_t*>(o), L.o, static_cast<const uint16_t*>(dO), L.dO, lse, p.dvec,
        p.lse2, N, n_pad, Hq, rows_pad, p.scale,
        (p.dq_fp32 && !accumulate) ? static_cast<float*>(dq) : nullptr, L.dq);
    if (int st = launch_status("bwd_preprocess_kernel")) return st;
  }
  if (stages & FA_B200_STAGE_DKDV) {
    bwd_dkdv_kernel<D, BF><<<dim3(static_cast<unsigned>(BHkv), nq128), DkdvCfg<D>::THREADS,
                         DkdvCfg<D>::SMEM, stream>>>(tq, tk, tv, tdo, p);
    if (int st = launch_status("bwd_dkdv_kernel")) return st;
  }
  if (stages & FA_B200_STAGE_FUSED) {
    // dQ (fp32) as 32-row x 32-column boxes for the TMA reduce-adds
    CUtensorMap tdq;
    if (!make_map4(&tdq, dq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, Hq, B, L.dq, 32))
      return FA_B200_ERR_TENSOR_MAP;
    if (BHkv * static_cast<uint64_t>(nq128) * 16 > 0x7fffffffull) return FA_B200_ERR_TOO_LARGE;
    // A GQA group may be split over several CTAs, which add their partial
    // dK/dV into an fp32 accumulator in the workspace (when the caller sized
    // it with fa_b200_backward_workspace_bytes_gqa). With too few (batch,
    // kv-head) x key-block CTAs to fill the GPU the split is chosen by waves;
    // otherwise by replaying the dispatch.
    const size_t rows_bytes = 2 * sizeof(float) * static_cast<size_t>(rows_pad);
    const size_t acc_bytes = 2 * sizeof(float) * static_cast<size_t>(BHkv) * N * D;
    const FusedChoice fc = choose_fused(BHkv, nq128, p.group, causal != 0, N, D, sms, accumulate,
                                        accumulate || ws_bytes >= rows_bytes + acc_bytes);
    p.gsplit = fc.gsplit;
    p.gper = fc.gper;
    p.head_group = fc.head_group;
    // fp32 dK / dV accumulators (32-row boxes) for the reduce-add epilogue: the
    // caller's dk/dv when accumulating, else the workspace of a split group
    CUtensorMap tdka = tdq, tdva = tdq;   // unused by the 16-bit store epilogue
    if (accumulate) {
      if (!make_map4(&tdka, dk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, Hkv, B, L.dk, 32) ||
          !make_map4(&tdva, dv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, Hkv, B, L.dv, 32))
        return FA_B200_ERR_TENSOR_MAP;
    } else if (p.gsplit > 1) {
      p.dkv_reduce = 1;
      p.dkv_acc = ws + 2 * rows_pad;
      if (cudaMemsetAsync(p.dkv_acc, 0, acc_bytes, stream) != cudaSuccess)
        return launch_status("the dK/dV accumulator memset");
      const Strides sacc = contiguous(Hkv, N, D);
      if (!make_map4(&tdka, p.dkv_acc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, Hkv, B, sacc, 32) ||
          !make_map4(&tdva, p.dkv_acc + BHkv * N * D, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, D, N, Hkv,
                     B, sacc, 32))
        return FA_B200_ERR_TENSOR_MAP;
    }
    CUtensorMap tdk = tdq, tdv = tdq;   // 16-bit dK / dV outputs, 64-column x 128-row boxes
    if (!accumulate && (!make_map4(&tdk, dk, dt, 2, D, N, Hkv, B, L.dk, 128) ||
                        !make_map4(&tdv, dv, dt, 2, D, N, Hkv, B, L.dv, 128)))
      return FA_B200_ERR_TENSOR_MAP;
    const uint64_t units = BHkv * static_cast<uint64_t>(nq128);
    bwd_fused_kernel<D, BF><<<static_cast<unsigned>(units * p.gsplit), FusedCfg<D>::THREADS,
                              FusedCfg<D>::SMEM, stream>>>(tq, tk, tv, tdo, tdq, tdka, tdva, tdk, tdv, p);
    if (int st = launch_status("bwd_fused_kernel")) return st;
    if (p.gsplit > 1 && !accumulate) {
      const long long total = 2ll * BHkv * N * (D / 8);
      bwd_dkv_convert_kernel<BF><<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
          p.dkv_acc, p.dk, L.dk, p.dv, L.dv, B, Hkv, N, D, total);
      if (int st = launch_status("bwd_dkv_convert_kernel")) return st;
    }
  }
  if (stages & FA_B200_STAGE_DQ) {
    bwd_dq_kernel<D, BF><<<dim3(static_cast<unsigned>(BH), nq128), DqCfg<D>::THREADS, DqCfg<D>::SMEM,
                       stream>>>(tq, tk, tv, tdo, p);
    if (int st = launch_status("bwd_dq_kernel")) return st;
  }
  return FA_B200_OK;
}

}  // namespace
}  // namespace fab

namespace fab {

// One 128x128x128 tile: c = A * B^T through the production layouts.
// Threads 0-127 read TMEM rows; thread 160 (warp 5) issues TMA; thread 128
// (warp 4) allocates TMEM and issues the MMAs.
__global__ void __launch_bounds__(192, 1)
    selftest_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                         const __half* a_raw, float* c, int a_mn, int b_mn, int a_by_threads,
                         int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t s_a = sbase, s_b = sbase + 32768;
  const uint32_t b_ld = sbase + 65536, b_mma = b_ld + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + 65536 + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5;
  const Ctl ctl{abort_flag, err};
  if (threadIdx.x == 0) {
    mbar_init(b_ld, 1);
    mbar_init(b_mma, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) tmem_alloc(smem_u32(tmem_slot), 256);
  if (a_by_threads == 1 && threadIdx.x < 128) {
    // A is [M][K]; thread m writes its row into the swizzled K-major layout.
    const int m = threadIdx.x;
    for (int c8 = 0; c8 < 16; ++c8) {
      const uint4 v = reinterpret_cast<const uint4*>(a_raw + m * 128)[c8];
      st_shared_v4(s_a + sw128_offset(m, c8, 128), v.x, v.y, v.z, v.w);
    }
    fence_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (a_by_threads == 2 && threadIdx.x < 128) {
    // A is [M][K]; thread m stores its row into TMEM lane m, columns 128..191,
    // two fp16 per 32-bit column (the A-from-TMEM operand layout).
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    for (int h = 0; h < 2; ++h) {
      uint32_t v[32];
      for (int i = 0; i < 32; ++i)
        v[i] = reinterpret_cast<const uint32_t*>(a_raw + threadIdx.x * 128)[32 * h + i];
      tmem_st32(tmem + 128 + 32 * h + lane_off, v);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 160) {
    mbar_arrive_expect_tx(b_ld, a_by_threads ? 32768 : 65536);
    for (int ch = 0; ch < 2; ++ch) {
      if (!a_by_threads) tma_load_3d(s_a + ch * 16384, &ta, b_ld, ch * 64, 0, 0);
      tma_load_3d(s_b + ch * 16384, &tb, b_ld, ch * 64, 0, 0);
    }
  }
  if (threadIdx.x == 128) {
    if (mbar_wait(b_ld, 0, ctl, kErrTimeoutMma)) {
      tc_fence_after();
      const uint32_t id = idesc_f16(128, 128, a_mn != 0, b_mn != 0);
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;  // K-major step
        const uint64_t da = a_mn ? sdesc_sw128(s_a + kk * 2048, 16384, 1024)
                                 : sdesc_sw128(s_a + koff, 16, 1024);
        const uint64_t db = b_mn ? sdesc_sw128(s_b + kk * 2048, 16384, 1024)
                                 : sdesc_sw128(s_b + koff, 16, 1024);
        if (a_by_threads == 2)
          mma_ts(tmem, tmem + 128 + kk * 8, db, id, kk > 0 ? 1u : 0u);
        else
          mma_ss(tmem, da, db, id, kk > 0 ? 1u : 0u);
      }
      mma_commit(b_mma);
    } else {
      drain_loads(b_ld, 1, 1);
    }
  }
  if (threadIdx.x < 128) {
    bool ok = mbar_wait(b_mma, 0, ctl, kErrTimeoutEpilogue);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      tc_fence_after();
      const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t v[32];
        tmem_ld32(tmem + 32 * ch + lane_off, v);
        tmem_ld_wait(v);
        for (int i = 0; i < 32; ++i) c[threadIdx.x * 128 + 32 * ch + i] = __uint_as_float(v[i]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) {
    __syncwarp();
    tmem_dealloc(tmem, 256);
  }
}

// Failure-detection self-test: thread 0 waits on a barrier nothing arrives on
// (phase 0 of a fresh mbarrier never completes), with the kernels' own bounded
// wait and a limit of limit_ns; it records kErrSelftest and returns. No TMA, MMA
// or tensor memory is involved, so nothing is left in flight.
__global__ void __launch_bounds__(32, 1) selftest_wait_kernel(unsigned long long limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    const Ctl ctl{&abort_flag, err};
    mbar_wait_limit(smem_u32(&bar), 0, ctl, kErrSelftest, limit_ns);
  }
}

}  // namespace fab

// Shared implementation of the contiguous and strided entry points.
namespace fab {
namespace {

Strides from_abi(fa_b200_strides st) { return Strides{st.batch, st.head, st.row}; }

int forward_impl(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                 int Hkv, int N, int D, int dtype, int causal, const FwdLayout& L, void* stream) {
  if (!q || !k || !v || !o || !lse) return FA_B200_ERR_NULL_POINTER;
  int st = check_shape(B, Hq, Hkv, N, D);
  if (st != FA_B200_OK) return st;
  if (dtype != FA_B200_DTYPE_FP16 && dtype != FA_B200_DTYPE_BF16) return FA_B200_ERR_DTYPE;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(lse) ||
      !strides_ok(L.q, 2) || !strides_ok(L.k, 2) || !strides_ok(L.v, 2) || !strides_ok(L.o, 2))
    return FA_B200_ERR_ALIGNMENT;
  int dev = 0, sms = 0;
  int* err = nullptr;
  st = device_setup(&dev, &err, &sms);
  if (st != FA_B200_OK) return st;
  auto s = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == FA_B200_DTYPE_BF16;
#define FAB_FWD(DD, BB) \
  launch_forward<DD, BB>(q, k, v, o, lse, B, Hq, Hkv, N, causal, L, sms, s, err)
  if (D == 64) return bf ? FAB_FWD(64, true) : FAB_FWD(64, false);
  return bf ? FAB_FWD(128, true) : FAB_FWD(128, false);
#undef FAB_FWD
}

// ws == nullptr: the built-in scratch of fa_b200_backward_noalloc.
int backward_impl(const void* q, const void* k, const void* v, const void* dO, const void* o,
                  const float* lse, void* dq, int dq_fp32, void* dk, void* dv, void* workspace,
                  size_t workspace_bytes, bool noalloc, int B, int Hq, int Hkv, int N, int D,
                  int dtype, int causal, int stages, const BwdLayout& L, void* stream) {
  if (stages == 0) stages = default_stages(dq_fp32);
  if (stages & ~(FA_B200_STAGE_ALL | FA_B200_STAGE_FUSED | FA_B200_STAGE_ACCUMULATE))
    return FA_B200_ERR_SHAPE;
  if ((stages & FA_B200_STAGE_FUSED) && (!dq_fp32 || (stages & (FA_B200_STAGE_DKDV | FA_B200_STAGE_DQ))))
    return FA_B200_ERR_SHAPE;
  // accumulating needs the fused stage (fp32 dq); dk/dv are then fp32
  const bool accumulate = (stages & FA_B200_STAGE_ACCUMULATE) != 0;
  if (accumulate && !(stages & FA_B200_STAGE_FUSED)) return FA_B200_ERR_SHAPE;
  if (!q || !k || !v || !dO || !o || !lse || !dq || !dk || !dv) return FA_B200_ERR_NULL_POINTER;
  int st = check_shape(B, Hq, Hkv, N, D);
  if (st != FA_B200_OK) return st;
  if (dtype != FA_B200_DTYPE_FP16 && dtype != FA_B200_DTYPE_BF16) return FA_B200_ERR_DTYPE;
  if (noalloc) {
    const size_t rows = static_cast<size_t>(B) * Hq * pad_rows(N);   // N <= kMaxN: no overflow
    if (rows > kNoAllocRows) {
      set_last_error(
          "fa_b200_backward_noalloc: B*Hq*roundup(N,128) = %zu query rows exceeds the built-in "
          "scratch of %zu rows (16 MiB); call fa_b200_backward with a caller-allocated workspace "
          "instead",
          rows, kNoAllocRows);
      return FA_B200_ERR_SCRATCH_LIMIT;
    }
  } else if (!workspace || workspace_bytes < fa_b200_backward_workspace_bytes(B, Hq, N)) {
    return FA_B200_ERR_WORKSPACE;
  }
  const void* ptrs[] = {q, k, v, dO, o, lse, dq, dk, dv};
  for (const void* ptr : ptrs)
    if (!aligned16(ptr)) return FA_B200_ERR_ALIGNMENT;
  if ((!noalloc && !aligned16(workspace)) || !strides_ok(L.q, 2) || !strides_ok(L.k, 2) ||
      !strides_ok(L.v, 2) || !strides_ok(L.dO, 2) || !strides_ok(L.o, 2) ||
      !strides_ok(L.dq, dq_fp32 ? 4 : 2) || !strides_ok(L.dk, accumulate ? 4 : 2) ||
      !strides_ok(L.dv, accumulate ? 4 : 2))
    return FA_B200_ERR_ALIGNMENT;
  int dev = 0, sms = 0;
  int* err = nullptr;
  st = device_setup(&dev, &err, &sms);
  if (st != FA_B200_OK) return st;
  float* ws = noalloc ? noalloc_scratch(dev) : static_cast<float*>(workspace);
  const size_t ws_bytes = noalloc ? 0 : workspace_bytes;
  if (!ws) return FA_B200_ERR_DEVICE;
  auto s = static_cast<cudaStream_t>(stream);
  const bool bf = dtype == FA_B200_DTYPE_BF16;
#define FAB_BWD(DD, BB)                                                                  \
  launch_backward<DD, BB>(q, k, v, dO, o, lse, dq, dq_fp32, dk, dv, ws, ws_bytes, B, Hq, Hkv, N, \
                          causal, stages, L, sms, s, err)
  if (D == 64) return bf ? FAB_BWD(64, true) : FAB_BWD(64, false);
  return bf ? FAB_BWD(128, true) : FAB_BWD(128, false);
#undef FAB_BWD
}

BwdLayout contiguous_bwd(int Hq, int Hkv, int N, int D) {
  const Strides sq = contiguous(Hq, N, D), skv = contiguous(Hkv, N, D);
  return BwdLayout{sq, skv, skv, sq, sq, sq, skv, skv};
}

}  // namespace
}  // namespace fab

// ===========================================================================
// extern "C" entry points
extern "C" {


int fa_b200_forward(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Hq,
                    int Hkv, int N, int D, int causal, int full_precision, void* stream) {
  (void)full_precision;
  const fab::Strides sq = fab::contiguous(Hq, N, D), skv = fab::contiguous(Hkv, N, D);
  return fab::forward_impl(q, k, v, o, lse, B, Hq, Hkv, N, D, FA_B200_DTYPE_FP16, causal,
                           fab::FwdLayout{sq, skv, skv, sq}, stream);
}

int fa_b200_forward_strided(const void* q, fa_b200_strides sq, const void* k, fa_b200_strides sk,
                            const void* v, fa_b200_strides sv, void* o, fa_b200_strides so,
                            float* lse, int B, int Hq, int Hkv, int N, int D, int dtype,
                            int causal, int full_precision, void* stream) {
  (void)full_precision;
  return fab::forward_impl(q, k, v, o, lse, B, Hq, Hkv, N, D, dtype, causal,
                           fab::FwdLayout{fab::from_abi(sq), fab::from_abi(sk), fab::from_abi(sv),
                                          fab::from_abi(so)},
                           stream);
}

int fa_b200_merge_partial(float* o, fa_b200_strides so, float* lse, fa_b200_strides slse,
                          const void* o_part, fa_b200_strides sop, const float* lse_part,
                          fa_b200_strides slp, int B, int H, int N, int D, int dtype,
                          void* stream) {
  if (!o || !lse || !o_part || !lse_part) return FA_B200_ERR_NULL_POINTER;
  if (D != 64 && D != 128) return FA_B200_ERR_HEAD_DIM;
  if (B < 1 || H < 1 || N < 1) return FA_B200_ERR_SHAPE;
  if (dtype != FA_B200_DTYPE_FP16 && dtype != FA_B200_DTYPE_BF16) return FA_B200_ERR_DTYPE;
  const fab::Strides a = fab::from_abi(so), p = fab::from_abi(sop);
  const fab::Strides la = fab::from_abi(slse), lp = fab::from_abi(slp);
  if (!fab::aligned16(o) || !fab::aligned16(o_part) || !fab::strides_ok(a, 4) ||
      !fab::strides_ok(p, 2) || la.b < 0 || la.h < 0 || la.n < 0 || lp.b < 0 || lp.h < 0 ||
      lp.n < 0)
    return FA_B200_ERR_ALIGNMENT;
  const long long total = static_cast<long long>(B) * H * N * (D / 8);
  if ((total + 255) / 256 > 0x7fffffffll) return FA_B200_ERR_TOO_LARGE;
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
  auto s = static_cast<cudaStream_t>(stream);
  if (dtype == FA_B200_DTYPE_BF16)
    fab::merge_partial_kernel<true><<<blocks, 256, 0, s>>>(
        o, a, lse, la, static_cast<const uint16_t*>(o_part), p, lse_part, lp, H, N, D, total);
  else
    fab::merge_partial_kernel<false><<<blocks, 256, 0, s>>>(
        o, a, lse, la, static_cast<const uint16_t*>(o_part), p, lse_part, lp, H, N, D, total);
  return fab::launch_status("merge_partial_kernel");
}

size_t fa_b200_backward_workspace_bytes(int B, int Hq, int N) {
  if (B < 1 || Hq < 1 || N < 1 || N > fab::kMaxN) return 0;
  // Dv and LSE*log2e for every query row, each head padded to a multiple of
  // 128 rows (a multiple of 512 bytes, so the total needs no rounding).
  return 2 * static_cast<size_t>(B) * Hq * fab::pad_rows(N) * sizeof(float);
}

size_t fa_b200_backward_workspace_bytes_gqa(int B, int Hq, int Hkv, int N, int D) {
  if (B < 1 || Hq < 1 || Hkv < 1 || N < 1 || D < 1 || N > fab::kMaxN) return 0;
  // the row values, then fp32 dK and dV accumulators for a split GQA group
  return fa_b200_backward_workspace_bytes(B, Hq, N) +
         2 * static_cast<size_t>(B) * Hkv * N * D * sizeof(float);
}

int fa_b200_backward_plan(int B, int Hq, int Hkv, int N, int D, int causal, size_t workspace_bytes,
                          int* gsplit, int* head_group) {
  if (!gsplit || !head_group) return FA_B200_ERR_NULL_POINTER;
  if (int st = fab::check_shape(B, Hq, Hkv, N, D)) return st;
  int dev = 0, sms = 0;
  int* err = nullptr;
  if (int st = fab::device_setup(&dev, &err, &sms)) return st;
  const uint64_t bhkv = static_cast<uint64_t>(B) * Hkv;
  const size_t rows_bytes = fa_b200_backward_workspace_bytes(B, Hq, N);
  const size_t acc_bytes = 2 * sizeof(float) * static_cast<size_t>(bhkv) * N * D;
  const fab::FusedChoice fc = fab::choose_fused(bhkv, (N + 127) / 128, Hq / Hkv, causal != 0, N, D,
                                                sms, false, workspace_bytes >= rows_bytes + acc_bytes);
  *gsplit = fc.gsplit;
  *head_group = fc.head_group;
  return FA_B200_OK;
}

int fa_b200_backward(const void* q, const void* k, const void* v, const void* dO, const void* o,
                     const float* lse, void* dq, int dq_fp32, void* dk, void* dv, void* workspace,
                     size_t workspace_bytes, int B, int Hq, int Hkv, int N, int D, int causal,
                     void* stream) {
  return fab::backward_impl(q, k, v, dO, o, lse, dq, dq_fp32, dk, dv, workspace, workspace_bytes,
                            false, B, Hq, Hkv, N, D, FA_B200_DTYPE_FP16, causal, 0,
                            fab::contiguous_bwd(Hq, Hkv, N, D), stream);
}

int fa_b200_backward_stages(const void* q, const void* k, const void* v, const void* dO,
                            const void* o, const float* lse, void* dq, int dq_fp32, void* dk,
                            void* dv, void* workspace, size_t workspace_bytes, int B, int Hq,
                            int Hkv, int N, int D, int causal, int stages, void* stream) {
  if (stages == 0) return FA_B200_ERR_SHAPE;
  return fab::backward_impl(q, k, v, dO, o, lse, dq, dq_fp32, dk, dv, workspace, workspace_bytes,
                            false, B, Hq, Hkv, N, D, FA_B200_DTYPE_FP16, causal, stages,
                            fab::contiguous_bwd(Hq, Hkv, N, D), stream);
}

int fa_b200_backward_strided(const void* q, fa_b200_strides sq, const void* k, fa_b200_strides sk,
                             const void* v, fa_b200_strides sv, const void* dO,
                             fa_b200_strides sdo, const void* o, fa_b200_strides so,
                             const float* lse, void* dq, fa_b200_strides sdq, int dq_fp32,
                             void* dk, fa_b200_strides sdk, void* dv, fa_b200_strides sdv,
                             void* workspace, size_t workspace_bytes, int B, int Hq, int Hkv,
                             int N, int D, int dtype, int causal, int stages, void* stream) {
  using fab::from_abi;
  return fab::backward_impl(q, k, v, dO, o, lse, dq, dq_fp32, dk, dv, workspace, workspace_bytes,
                            false, B, Hq, Hkv, N, D, dtype, causal, stages,
                            fab::BwdLayout{from_abi(sq), from_abi(sk), from_abi(sv), from_abi(sdo),
                                           from_abi(so), from_abi(sdq), from_abi(sdk),
                                           from_abi(sdv)},
                            stream);
}

size_t fa_b200_backward_noalloc_max_rows(void) { return fab::kNoAllocRows; }

int fa_b200_backward_noalloc(const void* q, const void* k, const void* v, const void* dO,
                             const void* o, const float* lse, void* dq, int dq_fp32, void* dk,
                             void* dv, int B, int Hq, int Hkv, int N, int D, int causal,
                             void* stream) {
  return fab::backward_impl(q, k, v, dO, o, lse, dq, dq_fp32, dk, dv, nullptr, 0, true, B, Hq,
                            Hkv, N, D, FA_B200_DTYPE_FP16, causal, 0,
                            fab::contiguous_bwd(Hq, Hkv, N, D), stream);
}

int fa_b200_device_error(int device, int reset) {
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return -1;
  if (cudaSetDevice(device) != cudaSuccess) return -1;
  int value = -1;
  if (cudaDeviceSynchronize() == cudaSuccess &&
      cudaMemcpyFromSymbol(&value, fab::g_device_error, sizeof(int)) == cudaSuccess && reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(fab::g_device_error, &zero, sizeof(int)) != cudaSuccess) value = -1;
  }
  cudaSetDevice(prev);
  return value;
}

int fa_b200_debug_tma_check(int device, unsigned long long* word, int reset) {
  if (!word) return FA_B200_ERR_NULL_POINTER;
#ifdef FAB_CHECK_TMA
  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return FA_B200_ERR_DEVICE;
  if (cudaSetDevice(device) != cudaSuccess) return FA_B200_ERR_DEVICE;
  int st = FA_B200_OK;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(word, fab::g_tma_check, sizeof(*word)) != cudaSuccess) {
    fab::launch_status("reading the TMA check word");   // records the message
    st = FA_B200_ERR_LAUNCH;
  } else if (reset) {
    const unsigned long long zero = 0;
    if (cudaMemcpyToSymbol(fab::g_tma_check, &zero, sizeof(zero)) != cudaSuccess) {
      fab::launch_status("clearing the TMA check word");
      st = FA_B200_ERR_LAUNCH;
    }
  }
  cudaSetDevice(prev);
  return st;
#else
  (void)device;
  (void)reset;
  *word = 0;
  return FA_B200_ERR_UNCHECKED_BUILD;
#endif
}

int fa_b200_device_error_async(int* host_word, void* stream) {
  if (!host_word) return FA_B200_ERR_NULL_POINTER;
  int dev = 0;
  int* err = nullptr;
  const int st = fab::device_setup(&dev, &err);
  if (st != FA_B200_OK) return st;
  if (cudaMemcpyAsync(host_word, err, sizeof(int), cudaMemcpyDeviceToHost,
                      static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return fab::launch_status("the device error word copy");
  return FA_B200_OK;
}

int fa_b200_selftest_wait(long long limit_ns, void* stream) {
  int dev = 0;
  int* err = nullptr;
  const int st = fab::device_setup(&dev, &err);
  if (st != FA_B200_OK) return st;
  const long long lim = std::min(std::max(limit_ns, 1000ll), 1000000000ll);
  fab::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<unsigned long long>(lim), err);
  return fab::launch_status("selftest_wait_kernel");
}

const char* fa_b200_last_error(void) { return fab::g_last_error; }

const char* fa_b200_status_string(int status) {
  switch (status) {
    case FA_B200_OK: return "ok";
    case FA_B200_ERR_NULL_POINTER: return "a required pointer is NULL";
    case FA_B200_ERR_HEAD_DIM: return "head dim must be 64 or 128";
    case FA_B200_ERR_SHAPE: return "bad shape: need B, N, Hkv >= 1 and Hq a multiple of Hkv";
    case FA_B200_ERR_ALIGNMENT: return "device pointers must be 16-byte aligned";
    case FA_B200_ERR_TENSOR_MAP: return "cuTensorMapEncodeTiled rejected a tensor";
    case FA_B200_ERR_LAUNCH: return "kernel launch failed";
    case FA_B200_ERR_WORKSPACE: return "workspace missing or too small";
    case FA_B200_ERR_DTYPE: return "dtype must be FA_B200_DTYPE_FP16 or FA_B200_DTYPE_BF16";
    case FA_B200_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case FA_B200_ERR_TOO_LARGE: return "problem exceeds a CUDA grid limit";
    case FA_B200_ERR_SCRATCH_LIMIT: return "problem exceeds the built-in scratch of the no-allocation backward";
    case FA_B200_ERR_UNCHECKED_BUILD: return "not a checked build (build with FA_B200_DEBUG=1 for the TMA checks)";
    default: return "unknown status";
  }
}

int fa_b200_selftest_gemm(const void* a, const void* b, float* c, int a_mn, int b_mn,
                          int a_by_threads, void* stream) {
  if (!a || !b || !c) return FA_B200_ERR_NULL_POINTER;
  if (!fab::aligned16(a) || !fab::aligned16(b) || !fab::aligned16(c)) return FA_B200_ERR_ALIGNMENT;
  if (a_by_threads && a_mn) return FA_B200_ERR_SHAPE;
  int dev = 0;
  int* err = nullptr;
  int st = fab::device_setup(&dev, &err);
  if (st != FA_B200_OK) return st;
  CUtensorMap ta, tb;
  if (!fab::make_map(&ta, a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 128, 128, 1, 128) ||
      !fab::make_map(&tb, b, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 128, 128, 1, 128))
    return FA_B200_ERR_TENSOR_MAP;
  constexpr int smem = 65536 + 64 + 1024;
  cudaFuncSetAttribute(fab::selftest_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  fab::selftest_gemm_kernel<<<1, 192, smem, static_cast<cudaStream_t>(stream)>>>(
      ta, tb, static_cast<const __half*>(a), c, a_mn, b_mn, a_by_threads, err);
  return cudaGetLastError() == cudaSuccess ? FA_B200_OK : FA_B200_ERR_LAUNCH;
}

}  // extern "C"
