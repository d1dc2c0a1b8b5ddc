// Error channel and small shared host utilities of the C ABI.
#include <initializer_list>
#include <atomic>
#include <cstring>

#include "common.cuh"

namespace pmb {

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
}

void clear_error() { g_last_error[0] = 0; }

static std::atomic<uint64_t> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int make_band_table(BandTable& t, int count, const int64_t* widths, const void* const* p0,
                    const void* const* p1, const void* const* p2, const char* name) {
  if (count <= 0 || count > kMaxBands) {
    set_error("%s: band count %d outside [1, %d]", name, count, kMaxBands);
    return PMB_ERR_INVALID_ARGUMENT;
  }
  if (widths == nullptr) {
    set_error("%s: band widths must not be NULL", name);
    return PMB_ERR_INVALID_ARGUMENT;
  }
  t.count = count;
  t.off[0] = 0;
  t.max_width = 0;
  for (int b = 0; b < count; ++b) {
    if (widths[b] <= 0) {
      set_error("%s: band %d has non-positive width %lld", name, b, (long long)widths[b]);
      return PMB_ERR_INVALID_ARGUMENT;
    }
    t.off[b + 1] = t.off[b] + widths[b];
    if (widths[b] > t.max_width) t.max_width = (int)widths[b];
    t.ptr0[b] = p0 ? p0[b] : nullptr;
    t.ptr1[b] = p1 ? p1[b] : nullptr;
    t.ptr2[b] = p2 ? p2[b] : nullptr;
  }
  for (int b = count; b < kMaxBands; ++b) {
    t.off[b + 1] = t.off[count];
    t.ptr0[b] = t.ptr1[b] = t.ptr2[b] = nullptr;
  }
  t.total = t.off[count];
  return PMB_OK;
}

// Per-translation-unit tcgen05 wait-timeout flags (umma.cuh).
unsigned int timeout_flag_gemm(int reset);
unsigned int timeout_flag_mask(int reset);
unsigned int timeout_flag_qkv(int reset);
unsigned int timeout_flag_ff(int reset);
unsigned int timeout_flag_rms(int reset);
unsigned int timeout_flag_band(int reset);
unsigned int timeout_flag_attn(int reset);

}  // namespace pmb

extern "C" {

unsigned int pmb_umma_timeout(int reset) {
  unsigned int first = 0;
  for (auto flag : {pmb::timeout_flag_gemm, pmb::timeout_flag_mask, pmb::timeout_flag_qkv, pmb::timeout_flag_ff, pmb::timeout_flag_rms,
                    pmb::timeout_flag_band, pmb::timeout_flag_attn}) {
    const unsigned int v = flag(reset);
    if (first == 0) first = v;
  }
  return first;
}

const char* pmb_version(void) { return "0.1.0"; }

const char* pmb_last_error(void) { return pmb::g_last_error; }

uint64_t pmb_launch_count(void) { return pmb::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
