// tune.cu — the GPU counterpart of the reference's GEMM autotuner (acfun.h:26-30,
// autotune.cpp:304-430).  The reference times KC/NC cache-blocking candidates on the host CPU
// and keeps the winners in ~/.cache/acfun/; here the tunable choice is the tcgen05 tile variant
// of a plain GEMM (gemm.cuh's numbering per family), measured with CUDA events on this GPU for
// a set of shape classes and kept in a text table:
//   $ACFUN_TUNE_CACHE, else $HOME/.cache/acfun/tile_table_<device name>_sm<cc>.txt
// `acfun_autotune()` measures and writes the table; later runs load it on first use;
// `ACFUN_AUTOTUNE=1` measures on first use when no table exists (the reference's switch).
// Without a table the built-in size heuristics choose, as they always did.  A table entry only
// selects among variants valid for the shape, so results stay those of the tested kernels.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "api_export.cuh"
#include "gemm.cuh"
#include "runtime.cuh"

namespace acf {
namespace {

std::mutex g_mu;
bool g_loaded = false;
std::unordered_map<uint32_t, int> g_table;  // shape class -> variant
std::string g_status = "static heuristics: no tile table loaded";
thread_local int g_forced = -1;

int lg2up(long long x) {
  int l = 0;
  while ((1LL << l) < x && l < 40) ++l;
  return l;
}

uint32_t class_key(TuneFamily f, int M, int N, int K) {
  return ((uint32_t)f << 24) | ((uint32_t)lg2up(M) << 16) | ((uint32_t)lg2up(N) << 8) |
         (uint32_t)lg2up(K);
}

std::string table_path() {
  if (const char* p = getenv("ACFUN_TUNE_CACHE"); p && *p) return p;
  const char* home = getenv("HOME");
  std::string dir = std::string(home && *home ? home : "/tmp") + "/.cache/acfun";
  cudaDeviceProp prop{};
  int dev = 0;
  cudaGetDevice(&dev);
  std::string name = "gpu";
  if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess) {
    name = prop.name;
    name += "_sm" + std::to_string(prop.major) + std::to_string(prop.minor);
  } else {
    cudaGetLastError();
  }
  for (char& ch : name)
    if (!((ch >= 'a' && ch <= 'z') || (ch >= 'A' && ch <= 'Z') || (ch >= '0' && ch <= '9')))
      ch = '_';
  return dir + "/tile_table_" + name + ".txt";
}

// "# acfun tile table v1" header, then one "family lgM lgN lgK variant us" line per class.
bool load_table(const std::string& path) {
  FILE* f = fopen(path.c_str(), "r");
  if (!f) return false;
  char line[256];
  std::unordered_map<uint32_t, int> t;
  bool header = false;
  while (fgets(line, sizeof(line), f)) {
    if (strncmp(line, "# acfun tile table v1", 21) == 0) {
      header = true;
      continue;
    }
    if (line[0] == '#' || line[0] == '\n') continue;
    int fam, lm, ln, lk, v;
    float us;
    if (sscanf(line, "%d %d %d %d %d %f", &fam, &lm, &ln, &lk, &v, &us) != 6) continue;
    if (fam < 0 || fam > 2 || v < 0 || v >= kTuneVariants[fam] || lm < 0 || lm > 40 || ln < 0 ||
        ln > 40 || lk < 0 || lk > 40)
      continue;
    t[((uint32_t)fam << 24) | ((uint32_t)lm << 16) | ((uint32_t)ln << 8) | (uint32_t)lk] = v;
  }
  fclose(f);
  if (!header) return false;
  g_table.swap(t);
  g_status = "tuned: " + std::to_string(g_table.size()) + " shape classes from " + path;
  return true;
}

}  // namespace

namespace {

// pseudo-random operand fill (the tensor pipe's power, hence its clock, depends on the data):
// bytes, or bf16 pairs uniform in [-1, 1)
__global__ void k_tune_fill(uint32_t* p, long long n, uint32_t seed, int bytes) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    uint32_t h = (uint32_t)i * 0x9E3779B1u ^ seed;
    h ^= h >> 15;
    h *= 0x2C1B3C6Du;
    h ^= h >> 12;
    if (bytes) {
      p[i] = h;
    } else {
      const float a = (float)(h & 0xFFFF) * (2.0f / 65536.0f) - 1.0f;
      const float b = (float)(h >> 16) * (2.0f / 65536.0f) - 1.0f;
      p[i] = (__float_as_uint(a) >> 16) | (__float_as_uint(b) & 0xFFFF0000u);
    }
  }
}

struct Shape {
  int M, N, K;
};
// shape classes measured per family: the BASELINE GEMMs, square sizes, a few wide / tall ones
// and the small-batch FC shapes
const Shape kShapes[3][7] = {
    {{512, 512, 512}, {1024, 1024, 1024}, {2048, 2048, 2048}, {4096, 4096, 4096},
     {256, 4096, 4096}, {256, 4096, 25088}, {8192, 512, 2048}},
    {{1024, 1024, 1024}, {2048, 2048, 2048}, {4096, 4096, 4096}, {8192, 2048, 2048},
     {0, 0, 0}, {0, 0, 0}, {0, 0, 0}},
    {{1024, 1024, 1024}, {2048, 2048, 2048}, {4096, 4096, 4096}, {8192, 8192, 4096},
     {0, 0, 0}, {0, 0, 0}, {0, 0, 0}}};

void* dev_alloc(size_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

// Mean microseconds of one launch of variant v (2 warm-ups, then 5 timed on the call's
// stream), or a negative value when it could not run.
float time_variant(Call& c, TuneFamily f, int v, const Shape& s, const Operand& A,
                   const Operand& B, void* C) {
  EpiParams ep{};
  ep.C = C;
  ep.ldc = s.N;
  const GemmKind kind = f == TuneFamily::F32 ? GemmKind::BF16X3
                        : f == TuneFamily::BF16 ? GemmKind::BF16 : GemmKind::I8U;
  const Epi epi = f == TuneFamily::I8 ? Epi::S32 : Epi::F32_BIAS;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
    cudaGetLastError();
    return -1.0f;
  }
  g_forced = v;
  bool ok = true;
  for (int w = 0; w < 2 && ok; ++w) ok = gemm_launch(c, kind, epi, A, B, s.M, s.N, s.K, ep);
  cudaEventRecord(e0, c.stream());
  for (int r = 0; r < 5 && ok; ++r) ok = gemm_launch(c, kind, epi, A, B, s.M, s.N, s.K, ep);
  cudaEventRecord(e1, c.stream());
  g_forced = -1;
  float ms = -1.0f;
  if (ok && cudaEventSynchronize(e1) == cudaSuccess && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess)
    ms = ms * 1000.0f / 5.0f;
  else
    ms = -1.0f;
  cudaGetLastError();
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  return ms;
}

// Measures every family's shape classes (caller holds g_mu), fills g_table and writes it.
bool run_tuning(Call& c, const std::string& path) {
  std::unordered_map<uint32_t, int> t;
  std::string lines;
  for (int fi = 0; fi < 3 && c.ok(); ++fi) {
    const TuneFamily f = (TuneFamily)fi;
    for (const Shape& s : kShapes[fi]) {
      if (s.M == 0) continue;
      const int ea = f == TuneFamily::I8 ? 1 : 2;                // bytes per element
      const int na = f == TuneFamily::F32 ? 2 : 1;               // hi / lo copies
      const size_t ab = (size_t)na * s.M * s.K * ea, bb = (size_t)na * s.K * s.N * ea;
      const size_t cb = (size_t)s.M * s.N * 4;
      void* a = dev_alloc(ab);
      void* b = dev_alloc(bb);
      void* cc = dev_alloc(cb);
      if (a && b && cc) {
        k_tune_fill<<<1184, 256, 0, c.stream()>>>((uint32_t*)a, (long long)(ab / 4), 0x1234u + fi,
                                                  f == TuneFamily::I8);
        k_tune_fill<<<1184, 256, 0, c.stream()>>>((uint32_t*)b, (long long)(bb / 4), 0x9876u + fi,
                                                  f == TuneFamily::I8);
        Operand A, B;
        A.p = a;
        A.ld = s.K;
        A.op_stride = (long long)s.M * s.K;
        B.p = b;
        B.ld = s.N;
        B.op_stride = (long long)s.K * s.N;
        int best = -1;
        float best_us = 0.0f;
        for (int v = 0; v < kTuneVariants[fi]; ++v) {
          if (!tune_variant_valid(f, v, s.M, s.N, s.K)) continue;
          const float us = time_variant(c, f, v, s, A, B, cc);
          if (us > 0.0f && (best < 0 || us < best_us)) {
            best = v;
            best_us = us;
          }
        }
        if (best >= 0) {
          t[class_key(f, s.M, s.N, s.K)] = best;
          char buf[96];
          snprintf(buf, sizeof(buf), "%d %d %d %d %d %.2f\n", fi, lg2up(s.M), lg2up(s.N),
                   lg2up(s.K), best, best_us);
          lines += buf;
        }
      }
      cudaStreamSynchronize(c.stream());
      cudaFree(a);
      cudaFree(b);
      cudaFree(cc);
      cudaGetLastError();
    }
  }
  if (t.empty()) {
    g_status = "static heuristics: tuning measured nothing";
    return false;
  }
  g_table.swap(t);
  g_status = "tuned: " + std::to_string(g_table.size()) + " shape classes measured";
  // the table file (directory created as needed); failing to write only loses the cache
  const size_t slash = path.rfind('/');
  if (slash != std::string::npos) {
    std::string dir = path.substr(0, slash);
    for (size_t i = 1; i <= dir.size(); ++i)
      if (i == dir.size() || dir[i] == '/') mkdir(dir.substr(0, i).c_str(), 0755);
  }
  if (FILE* fo = fopen(path.c_str(), "w")) {
    fprintf(fo, "# acfun tile table v1 (family lgM lgN lgK variant us; gemm.cuh numbering)\n%s",
            lines.c_str());
    fclose(fo);
    g_status += ", written to " + path;
  }
  return true;
}

}  // namespace

bool tune_variant_valid(TuneFamily f, int v, int M, int N, int K) {
  if (v < 0 || v >= kTuneVariants[(int)f] || M <= 0 || N <= 0 || K <= 0) return false;
  if (f == TuneFamily::F32 && v == 5)  // split-K: partials of M*N floats, >= 2 K ranges
    return K >= 1024 && (long long)M * N < (1LL << 31);
  return true;
}

int tune_variant(Call& c, TuneFamily f, int M, int N, int K) {
  if (g_forced >= 0) return g_forced;  // the tuner measuring (this thread, g_mu held)
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_loaded) {
    g_loaded = true;
    const std::string path = table_path();
    if (!load_table(path)) {
      g_status = "static heuristics: no tile table at " + path + " (acfun_autotune() measures one)";
      const char* e = getenv("ACFUN_AUTOTUNE");
      if (e && e[0] == '1') run_tuning(c, path);
    }
  }
  const auto it = g_table.find(class_key(f, M, N, K));
  return it == g_table.end() ? -1 : it->second;
}

void tune_force(int v) { g_forced = v; }

}  // namespace acf

using namespace acf;

// acfun.h:29 (autotune.cpp:421-425): measure the tile table on the current GPU and keep it.
extern "C" void acfun_autotune(void) {
  Call c("acfun_autotune");
  if (!c.ok()) return;
  std::lock_guard<std::mutex> g(g_mu);
  g_loaded = true;
  run_tuning(c, table_path());
  c.finish();
}

// acfun.h:30 (autotune.cpp:427-430)
extern "C" const char* acfun_tune_status(void) {
  static thread_local std::string s;
  {
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_loaded) {
      g_loaded = true;
      const std::string path = table_path();
      if (!load_table(path))
        g_status = "static heuristics: no tile table at " + path + " (acfun_autotune() measures one)";
    }
    s = g_status;
  }
  return s.c_str();
}
