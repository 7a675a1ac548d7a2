// Error state, device checks and group-layout resolution for libkvq.so.
#include <cstring>

#include "kvq_common.cuh"

namespace kvq {

static thread_local char g_err[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  return KVQ_OK;
}

int require_sm100() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("no CUDA device: %s", cudaGetErrorString(e));
    return KVQ_ERR_CUDA;
  }
  // cached per device; the compute capability never changes in a process
  static int cc_major[64];
  static bool have[64];
  if (dev < 0 || dev >= 64) {
    set_error("device ordinal %d out of range", dev);
    return KVQ_ERR_DEVICE;
  }
  if (!have[dev]) {
    int major = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) {
      set_error("cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
      return KVQ_ERR_CUDA;
    }
    cc_major[dev] = major;
    have[dev] = true;
  }
  if (cc_major[dev] != 10) {
    set_error("libkvq is built for sm_100a (B200); device %d is compute capability %d.x", dev,
              cc_major[dev]);
    return KVQ_ERR_DEVICE;
  }
  return KVQ_OK;
}

template <class L>
static bool matches(const int32_t* cb, int head_dim, int n_groups) {
  if (head_dim != 128 || n_groups != L::G) return false;
  for (int g = 0; g < L::G; ++g)
    for (int c = L::E[g]; c < L::E[g + 1]; ++c)
      if (cb[c] != g) return false;
  return true;
}

int resolve_layout(const int32_t* chan_band, int head_dim, int n_groups, GroupMap* map) {
  KVQ_REQUIRE(chan_band != nullptr, KVQ_ERR_ARG, "chan_band is NULL (it is a host array)");
  KVQ_REQUIRE(head_dim > 0 && head_dim <= kMaxHeadDim && head_dim % 8 == 0, KVQ_ERR_UNSUPPORTED,
              "head_dim %d unsupported (multiple of 8, at most %d)", head_dim, kMaxHeadDim);
  KVQ_REQUIRE(n_groups > 0 && n_groups <= kMaxGroups && n_groups <= head_dim, KVQ_ERR_ARG,
              "n_groups %d out of range", n_groups);
  bool seen[kMaxGroups] = {false};
  for (int c = 0; c < head_dim; ++c) {
    int g = chan_band[c];
    KVQ_REQUIRE(g >= 0 && g < n_groups, KVQ_ERR_ARG,
                "chan_band[%d] = %d is outside [0, %d)", c, g, n_groups);
    seen[g] = true;
    if (map) map->gid[c] = static_cast<uint8_t>(g);
  }
  for (int g = 0; g < n_groups; ++g)
    KVQ_REQUIRE(seen[g], KVQ_ERR_ARG, "group %d has no channel in chan_band", g);
  if (map)
    for (int c = head_dim; c < kMaxHeadDim; ++c) map->gid[c] = 0;
  if (matches<LayoutBands>(chan_band, head_dim, n_groups)) return kLayoutBands;
  if (matches<LayoutBands2>(chan_band, head_dim, n_groups)) return kLayoutBands2;
  if (matches<LayoutBands4>(chan_band, head_dim, n_groups)) return kLayoutBands4;
  if (matches<LayoutBlind32>(chan_band, head_dim, n_groups)) return kLayoutBlind32;
  if (matches<LayoutBlind64>(chan_band, head_dim, n_groups)) return kLayoutBlind64;
  return kLayoutGeneric;
}

}  // namespace kvq

extern "C" int kvq_abi_version(void) { return KVQ_ABI_VERSION; }

extern "C" const char* kvq_last_error(void) { return kvq::g_err; }
