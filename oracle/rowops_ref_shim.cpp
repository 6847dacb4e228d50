// TEST INFRASTRUCTURE — a C-ABI shim over the reference's row-ops oracle
// (phoenix367/cormorant kernels/rowops_rtl/tb/verilator/rowops_ref.h, compiled
// from where it lies by oracle/Makefile into oracle/_ref/).  Runs one job (or
// a chain) on a flat memory image, as the RTL testbench does, and applies the
// job's writes to the image.  Used only by tests to check the numpy
// restatement (oracle/spec.py) and the GPU kernels.
#include <cstddef>
#include <cstdint>

#include "rowops_ref.h"

extern "C" int ro_ref_run(uint8_t* mem, size_t len, const uint64_t* r, int njobs) {
  // r: per job 20 words: op n c1 c2 a a_s1 a_s2 b b_s1 b_s2 c c_s1 c_s2 p eps aux bq_sh win_lo win_hi (reserved)
  ro::Mem m{[&](uint64_t a) -> uint8_t { return a < len ? mem[a] : 0; }};
  ro::PState ps;
  std::vector<ro::Job> jobs;
  for (int k = 0; k < njobs; k++) {
    const uint64_t* w = r + 20 * k;
    ro::Job j;
    j.op = (uint32_t)w[0]; j.n = (uint32_t)w[1]; j.c1 = (uint32_t)w[2]; j.c2 = (uint32_t)w[3];
    j.a = w[4]; j.a_s1 = (uint32_t)w[5]; j.a_s2 = (uint32_t)w[6];
    j.b = w[7]; j.b_s1 = (uint32_t)w[8]; j.b_s2 = (uint32_t)w[9];
    j.c = w[10]; j.c_s1 = (uint32_t)w[11]; j.c_s2 = (uint32_t)w[12];
    j.p = w[13]; j.eps = w[14]; j.aux = (uint32_t)w[15]; j.bq_sh = (uint32_t)w[16];
    j.win_lo = (uint32_t)w[17]; j.win_hi = (uint32_t)w[18];
    jobs.push_back(j);
  }
  auto img = ro::run_chain(jobs, m, &ps);
  for (auto& kv : img) {
    if (kv.first >= len) return -1;
    mem[kv.first] = kv.second;
  }
  return 0;
}
