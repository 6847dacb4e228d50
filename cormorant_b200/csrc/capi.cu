// Library plumbing: errors, the device check, the per-device scratch and the
// per-device unit tables, and the host-side helper entry points.
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "corm_common.cuh"
#include "postop.cuh"

namespace corm {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_err, sizeof g_err, fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CORM_ECUDA, "%s: %s", where, cudaGetErrorString(e));
  return CORM_OK;
}

static std::mutex g_mu;
static const int kMaxDev = 64;
static int g_dev_ok[kMaxDev];  // 0 unknown, 1 sm_100, -1 other

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(CORM_ECUDA, "no CUDA device");
  if (dev < 0 || dev >= kMaxDev) return fail(CORM_EDEVICE, "device index %d", dev);
  if (g_dev_ok[dev] == 0) {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return fail(CORM_ECUDA, "device properties");
    g_dev_ok[dev] = (p.major == 10 && p.minor == 0) ? 1 : -1;
  }
  if (g_dev_ok[dev] < 0) return fail(CORM_EDEVICE, "libcorm_b200 is built for sm_100a only");
  return CORM_OK;
}

struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
};
static Scratch g_scratch[kMaxDev];

void* scratch(size_t bytes, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  Scratch& s = g_scratch[dev];
  if (s.bytes >= bytes && s.ptr) return s.ptr;
  // grow: wait for users of the old block on this stream, then replace it
  if (s.ptr) {
    cudaStreamSynchronize(stream);
    cudaDeviceSynchronize();
    cudaFree(s.ptr);
    s.ptr = nullptr;
    s.bytes = 0;
  }
  size_t want = bytes < (64u << 20) ? (64u << 20) : bytes + (bytes >> 3);
  if (cudaMalloc(&s.ptr, want) != cudaSuccess) {
    cudaGetLastError();
    s.ptr = nullptr;
    set_error("scratch: cudaMalloc of %zu bytes failed", want);
    return nullptr;
  }
  s.bytes = want;
  return s.ptr;
}

static DeviceTables g_tables[kMaxDev];
static bool g_tables_ok[kMaxDev];

const DeviceTables* tables() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_tables_ok[dev]) return &g_tables[dev];
  DeviceTables t{};
  std::vector<int16_t> act(65536);
  for (int a = 4; a <= 6; a++) {
    build_act_table(a, 0, act.data());
    void* p = nullptr;
    if (cudaMalloc(&p, 65536 * 2) != cudaSuccess ||
        cudaMemcpy(p, act.data(), 65536 * 2, cudaMemcpyHostToDevice) != cudaSuccess) {
      set_error("tables: upload failed");
      return nullptr;
    }
    t.act[a] = (const int16_t*)p;
  }
  std::vector<int32_t> tab(4096);
  build_smx_tab(tab.data());
  void* p = nullptr;
  if (cudaMalloc(&p, 4096 * 4) != cudaSuccess ||
      cudaMemcpy(p, tab.data(), 4096 * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    set_error("tables: upload failed");
    return nullptr;
  }
  t.smx_tab = (const int32_t*)p;
  std::vector<uint8_t> img(65536);
  build_rowops_image(img.data());
  if (cudaMalloc(&p, 65536) != cudaSuccess || cudaMemcpy(p, img.data(), 65536, cudaMemcpyHostToDevice) != cudaSuccess) {
    set_error("tables: upload failed");
    return nullptr;
  }
  t.ro_sig = (uint64_t*)p;
  t.ro_rsq = (uint32_t*)((uint8_t*)p + 32768);
  g_tables[dev] = t;
  g_tables_ok[dev] = true;
  return &g_tables[dev];
}

// ---------------------------------------------------------------- tracing
static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_prof_on{0};
struct ProfRec {
  const char* name;
  cudaEvent_t a, b;
};
static std::mutex g_prof_mu;
static std::vector<ProfRec> g_prof;

ProfScope::ProfScope(const char* n, cudaStream_t s) : name(n), stream(s), slot(-1) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  ProfRec r{n, nullptr, nullptr};
  if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return;
  cudaEventRecord(r.a, s);
  std::lock_guard<std::mutex> lk(g_prof_mu);
  slot = (int)g_prof.size();
  g_prof.push_back(r);
}

ProfScope::~ProfScope() {
  if (slot < 0) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  cudaEventRecord(g_prof[slot].b, stream);
}

int make_postop(const void* pp, PostOp& out) {
  out = PostOp{};
  if (!pp) return CORM_OK;
  const corm_postop* p = (const corm_postop*)pp;
  if (!p->b) return fail(CORM_EINVAL, "postop: null operand");
  if (p->op > 2) return fail(CORM_EINVAL, "postop: op %u (0 ADD, 1 SUB, 2 MUL)", p->op);
  if (p->act > 6) return fail(CORM_EINVAL, "postop: act %u", p->act);
  if (p->b_mode > 2) return fail(CORM_EINVAL, "postop: b_mode %u", p->b_mode);
  if (p->act >= 4) {
    const DeviceTables* tb = tables();
    if (!tb) return CORM_ECUDA;
    out.table = tb->act[p->act];
  }
  out.b = p->b;
  out.op = p->op;
  out.act = p->act;
  out.alpha = p->alpha;
  out.b_mode = p->b_mode;
  out.rev = p->b_is_first ? 1u : 0u;
  return CORM_OK;
}

}  // namespace corm

extern "C" {

uint64_t corm_launch_count(void) { return corm::g_launches.load(); }

int corm_profile_enable(int on) {
  corm::g_prof_on.store(on ? 1 : 0);
  return CORM_OK;
}

int corm_profile_read(corm_profile_entry* out, int max_entries, int* n_out) {
  std::vector<corm::ProfRec> recs;
  {
    std::lock_guard<std::mutex> lk(corm::g_prof_mu);
    recs.swap(corm::g_prof);
  }
  int n = 0;
  for (auto& r : recs) {
    float ms = 0.f;
    cudaEventSynchronize(r.b);
    cudaEventElapsedTime(&ms, r.a, r.b);
    int i = 0;
    while (i < n && std::strncmp(out[i].name, r.name, sizeof out[i].name) != 0) i++;
    if (i == n && n < max_entries) {
      std::memset(&out[n], 0, sizeof out[n]);
      std::strncpy(out[n].name, r.name, sizeof out[n].name - 1);
      n++;
    }
    if (i < n) {
      out[i].launches++;
      out[i].total_ms += ms;
      if (ms > out[i].max_ms) out[i].max_ms = ms;
    }
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  if (n_out) *n_out = n;
  return corm::cuda_status("corm_profile_read");
}


int corm_act_table(uint32_t act, uint32_t alpha, int16_t* out65536) {
  if (!out65536 || act > 6) return corm::fail(CORM_EINVAL, "corm_act_table: bad argument");
  corm::build_act_table((int)act, alpha, out65536);
  return CORM_OK;
}

int corm_smx_table(int32_t* out4096) {
  if (!out4096) return corm::fail(CORM_EINVAL, "corm_smx_table: null output");
  corm::build_smx_tab(out4096);
  return CORM_OK;
}

int corm_rowops_table_image(uint8_t* out65536) {
  if (!out65536) return corm::fail(CORM_EINVAL, "corm_rowops_table_image: null output");
  corm::build_rowops_image(out65536);
  return CORM_OK;
}

int corm_bind_device(int device) {
  if (cudaSetDevice(device) != cudaSuccess) return corm::cuda_status("corm_bind_device");
  return CORM_OK;
}

const char* corm_version(void) { return "cormorant_b200 0.1 (sm_100a)"; }
const char* corm_last_error(void) { return corm::g_err; }


}  // extern "C"

extern "C" int corm_stream_done(corm_stream_t stream) {
  const cudaError_t e = cudaStreamQuery((cudaStream_t)stream);
  if (e == cudaSuccess) return 1;
  if (e == cudaErrorNotReady) return 0;
  return corm::cuda_status("corm_stream_done");
}
