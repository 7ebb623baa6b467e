// Fused elementwise code generation: one straight-line CUDA kernel per
// elementwise program (kvm_ew_program -- the kernel dialect's add sub mul div
// max min neg exp log sqrt rsqrt abs, cmp.*, cast.*, as the graph executor
// strings a chain of them together), compiled at run time by NVRTC for
// sm_100a and cached.
//
// Why generate code: an interpreter keeps its registers in an array indexed
// at run time (local memory) and recomputes 64-bit (i / div) % size for every
// load of every element. The generated kernel has the program's registers in
// real registers, the broadcast divisors as compile-time constants, and moves
// 8 consecutive output elements per thread with 16-byte loads and stores, so
// it streams at HBM speed for any chain length that fits the program limits.
//
// Layout per input, from (in_size, in_div) (element i reads
// (i / in_div) % in_size):
//   in_div == 1          a contiguous run: 8 lanes load 16 B at i % in_size
//                        (in_size a constant: the modulo is a multiply)
//   in_div % 8 == 0      one value per 8 outputs, broadcast to the lanes
//   otherwise            per-element indexing (the 1-element-per-thread form)
// The 8-wide form needs n % 8 == 0, 16-byte aligned pointers for contiguous
// inputs and the output, and in_size % 8 == 0 for contiguous inputs.
//
// NVRTC is opened at run time (libnvrtc.so.12). Generated code uses no CUDA
// header: conversions are PTX cvt instructions; math calls are the CUDA math
// API functions NVRTC provides (expf, logf, sqrtf, rsqrtf, __fdiv_rn,
// __frcp_rn), the same calls the interpreter makes, so both paths agree bit
// for bit.
#include <dlfcn.h>
#include <nvrtc.h>

#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

#include "ew_jit.h"
#include "runtime.h"

namespace kvm {
namespace {

struct Nvrtc {
  nvrtcResult (*Create)(nvrtcProgram*, const char*, const char*, int, const char* const*,
                        const char* const*) = nullptr;
  nvrtcResult (*Compile)(nvrtcProgram, int, const char* const*) = nullptr;
  nvrtcResult (*LogSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*Log)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*CubinSize)(nvrtcProgram, size_t*) = nullptr;
  nvrtcResult (*Cubin)(nvrtcProgram, char*) = nullptr;
  nvrtcResult (*Destroy)(nvrtcProgram*) = nullptr;
  const char* (*ErrorString)(nvrtcResult) = nullptr;
  std::string error;
};

template <typename F>
bool sym(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  return *out != nullptr;
}

const Nvrtc* nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      n.error = std::string("cannot open libnvrtc.so.12: ") + dlerror();
      return;
    }
    const bool ok = sym(h, "nvrtcCreateProgram", &n.Create) &&
                    sym(h, "nvrtcCompileProgram", &n.Compile) &&
                    sym(h, "nvrtcGetProgramLogSize", &n.LogSize) &&
                    sym(h, "nvrtcGetProgramLog", &n.Log) &&
                    sym(h, "nvrtcGetCUBINSize", &n.CubinSize) &&
                    sym(h, "nvrtcGetCUBIN", &n.Cubin) &&
                    sym(h, "nvrtcDestroyProgram", &n.Destroy) &&
                    sym(h, "nvrtcGetErrorString", &n.ErrorString);
    if (!ok) n.error = "libnvrtc.so.12 lacks a required symbol";
  });
  if (!n.error.empty()) {
    fail(KVM_ERR_UNSUPPORTED, n.error);
    return nullptr;
  }
  return &n;
}

constexpr int kVec = 8;        // outputs per thread in the wide form
constexpr int kThreads = 256;  // threads per block

enum Access { kRun, kSpread, kElem };  // contiguous / one per vector / per element

struct Shape {
  int vec = 1;         // 8 or 1
  bool wide = false;   // 64-bit indices (n >= 2^31)
  Access access[KVM_EW_MAX_INPUTS];
};

Shape choose(const kvm_ew_program& p, const kvm_ew_inputs& in, const void* out, int64_t n) {
  Shape s;
  s.wide = n >= (int64_t(1) << 31);
  bool vec_ok = n % kVec == 0 && aligned16(out);
  for (int i = 0; i < p.n_inputs; ++i) {
    if (p.in_size[i] == 1) {
      s.access[i] = kSpread;  // a scalar
    } else if (p.in_div[i] == 1) {
      s.access[i] = kRun;
      if (p.in_size[i] % kVec != 0 || !aligned16(in.ptr[i])) vec_ok = false;
    } else if (p.in_div[i] % kVec == 0) {
      s.access[i] = kSpread;
    } else {
      s.access[i] = kElem;
      vec_ok = false;
    }
  }
  s.vec = vec_ok ? kVec : 1;
  if (s.vec == 1)
    for (int i = 0; i < p.n_inputs; ++i) s.access[i] = kElem;
  return s;
}

// Cache key: everything the generated source depends on.
std::string key_of(const kvm_ew_program& p, const Shape& s) {
  std::ostringstream k;
  k << p.n_inputs << ',' << p.n_instr << ',' << p.out_reg << ',' << p.out_dtype << ';'
    << s.vec << s.wide << ';';
  for (int i = 0; i < p.n_inputs; ++i)
    k << p.in_dtype[i] << ':' << p.in_size[i] << ':' << p.in_div[i] << ':' << s.access[i]
      << ';';
  for (int i = 0; i < p.n_instr; ++i)
    k << int(p.op[i]) << '.' << int(p.a[i]) << '.' << int(p.b[i]) << '.' << int(p.dst[i])
      << ' ';
  return k.str();
}

const char* kPrelude = R"(
typedef unsigned int u32;
typedef unsigned long long u64;
typedef unsigned short u16;
struct alignas(16) q4 { u32 x, y, z, w; };
static __device__ __forceinline__ float bf2f(u32 h) { return __uint_as_float(h << 16); }
static __device__ __forceinline__ float h2f(u32 h) {
  float f; u16 s = (u16)h; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(s)); return f; }
static __device__ __forceinline__ u32 f2bf(float f) {
  u16 h; asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
static __device__ __forceinline__ u32 f2h(float f) {
  u16 h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
static __device__ __forceinline__ u32 pack_bf(float lo, float hi) {
  u32 r; asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo)); return r; }
static __device__ __forceinline__ u32 pack_h(float lo, float hi) {
  u32 r; asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo)); return r; }
static __device__ __forceinline__ float ld1(const void* p, u64 i, int dt) {
  switch (dt) {
    case 0: return bf2f(((const u16*)p)[i]);
    case 2: return h2f(((const u16*)p)[i]);
    case 3: return (float)((const int*)p)[i];
    default: return ((const float*)p)[i];
  }
}
)";

// The 8 lanes of a contiguous input at element index `idx` (a multiple of 8).
void emit_load_run(std::ostringstream& o, const std::string& t, int dt, int slot,
                   const std::string& idx) {
  if (dt == KVM_EW_BF16 || dt == KVM_EW_F16) {
    const char* cv = dt == KVM_EW_BF16 ? "bf2f" : "h2f";
    o << "  { const q4 q = *(const q4*)((const u16*)in" << slot << " + " << idx << ");\n"
      << "    const u32 w[4] = {q.x, q.y, q.z, q.w};\n"
      << "#pragma unroll\n    for (int k = 0; k < 4; ++k) { " << t << "[2*k] = " << cv
      << "(w[k] & 0xFFFFu); " << t << "[2*k+1] = " << cv << "(w[k] >> 16); } }\n";
  } else {
    const char* ty = dt == KVM_EW_I32 ? "int" : "float";
    o << "  { const q4 q0 = *(const q4*)((const " << ty << "*)in" << slot << " + " << idx
      << "), q1 = *(const q4*)((const " << ty << "*)in" << slot << " + " << idx
      << " + 4);\n"
      << "    const u32 w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};\n"
      << "#pragma unroll\n    for (int k = 0; k < 8; ++k) " << t << "[k] = "
      << (dt == KVM_EW_I32 ? "(float)(int)w[k]" : "__uint_as_float(w[k])") << "; }\n";
  }
}

std::string unary(int op, const std::string& a) {
  switch (op) {
    case KVM_EW_NEG: return "-" + a;
    case KVM_EW_EXP: return "expf(" + a + ")";
    case KVM_EW_LOG: return "logf(" + a + ")";
    case KVM_EW_SQRT: return "sqrtf(" + a + ")";
    case KVM_EW_RSQRT: return "rsqrtf(" + a + ")";
    case KVM_EW_ABS: return "fabsf(" + a + ")";
    case KVM_EW_RCP: return "__frcp_rn(" + a + ")";
    case KVM_EW_ROUND_BF16: return "bf2f(f2bf(" + a + "))";
    case KVM_EW_ROUND_F16: return "h2f(f2h(" + a + "))";
    case KVM_EW_TRUNC_I32: return "truncf(" + a + ")";
    default: return "";
  }
}

std::string binary(int op, const std::string& a, const std::string& b) {
  switch (op) {
    case KVM_EW_ADD: return a + " + " + b;
    case KVM_EW_SUB: return a + " - " + b;
    case KVM_EW_MUL: return a + " * " + b;
    case KVM_EW_DIV: return "__fdiv_rn(" + a + ", " + b + ")";
    case KVM_EW_MAX: return "fmaxf(" + a + ", " + b + ")";
    case KVM_EW_MIN: return "fminf(" + a + ", " + b + ")";
    case KVM_EW_CMP_EQ: return "(" + a + " == " + b + " ? 1.f : 0.f)";
    case KVM_EW_CMP_NE: return "(" + a + " != " + b + " ? 1.f : 0.f)";
    case KVM_EW_CMP_LT: return "(" + a + " < " + b + " ? 1.f : 0.f)";
    case KVM_EW_CMP_LE: return "(" + a + " <= " + b + " ? 1.f : 0.f)";
    case KVM_EW_CMP_GT: return "(" + a + " > " + b + " ? 1.f : 0.f)";
    case KVM_EW_CMP_GE: return "(" + a + " >= " + b + " ? 1.f : 0.f)";
    default: return "";
  }
}

std::string source_of(const kvm_ew_program& p, const Shape& s) {
  std::ostringstream o;
  const int V = s.vec;
  const char* ix = s.wide ? "u64" : "u32";
  o << kPrelude << "extern \"C\" __global__ void __launch_bounds__(" << kThreads
    << ") kvm_ew(";
  for (int i = 0; i < p.n_inputs; ++i) o << "const void* __restrict__ in" << i << ", ";
  o << "void* __restrict__ out, u64 nvec) {\n"
    << "  const " << ix << " v = (" << ix << ")blockIdx.x * " << kThreads
    << "u + threadIdx.x;\n  if (v >= nvec) return;\n"
    << "  const " << ix << " i0 = v * " << V << "u;\n";
  std::string cur[KVM_EW_MAX_REGS];  // register -> the variable that holds it
  auto reg = [&](int r) { return cur[r].empty() ? std::string("zero") : cur[r]; };
  o << "  float zero[" << V << "];\n#pragma unroll\n  for (int k = 0; k < " << V
    << "; ++k) zero[k] = 0.f;\n";
  for (int st = 0; st < p.n_instr; ++st) {
    const int op = p.op[st];
    const std::string t = "t" + std::to_string(st);
    o << "  float " << t << "[" << V << "];\n";
    if (op == KVM_EW_LOAD) {
      const int slot = p.a[st];
      const int dt = p.in_dtype[slot];
      const int64_t size = p.in_size[slot], div = p.in_div[slot];
      const std::string sz = std::to_string(size) + (s.wide ? "ull" : "u");
      const std::string dv = std::to_string(div) + (s.wide ? "ull" : "u");
      if (s.access[slot] == kRun) {
        // i0 % size is a multiple of 8 (size % 8 == 0), so the 8 lanes are one run
        emit_load_run(o, t, dt, slot, "(i0 % " + sz + ")");
      } else if (s.access[slot] == kSpread) {
        const std::string idx = size == 1 ? std::string("0") : "((i0 / " + dv + ") % " + sz + ")";
        o << "  { const float x = ld1(in" << slot << ", " << idx << ", " << dt
          << ");\n#pragma unroll\n    for (int k = 0; k < " << V << "; ++k) " << t
          << "[k] = x; }\n";
      } else {
        o << "#pragma unroll\n  for (int k = 0; k < " << V << "; ++k) " << t << "[k] = ld1(in"
          << slot << ", ((i0 + k) / " << dv << ") % " << sz << ", " << dt << ");\n";
      }
    } else {
      const std::string a = reg(p.a[st]) + "[k]", b = reg(p.b[st]) + "[k]";
      std::string e = unary(op, a);
      if (e.empty()) e = binary(op, a, b);
      o << "#pragma unroll\n  for (int k = 0; k < " << V << "; ++k) " << t << "[k] = " << e
        << ";\n";
    }
    cur[p.dst[st]] = t;
  }
  const std::string r = reg(p.out_reg);
  switch (p.out_dtype) {
    case KVM_EW_BF16:
    case KVM_EW_F16: {
      const char* pk = p.out_dtype == KVM_EW_BF16 ? "pack_bf" : "pack_h";
      const char* one = p.out_dtype == KVM_EW_BF16 ? "f2bf" : "f2h";
      if (V == kVec)
        o << "  q4 q; q.x = " << pk << "(" << r << "[0], " << r << "[1]); q.y = " << pk << "("
          << r << "[2], " << r << "[3]); q.z = " << pk << "(" << r << "[4], " << r
          << "[5]); q.w = " << pk << "(" << r << "[6], " << r << "[7]);\n"
          << "  *(q4*)((u16*)out + i0) = q;\n";
      else
        o << "  ((u16*)out)[i0] = (u16)" << one << "(" << r << "[0]);\n";
      break;
    }
    case KVM_EW_I32:
      o << "#pragma unroll\n  for (int k = 0; k < " << V << "; ++k) ((int*)out)[i0 + k] = (int)"
        << r << "[k];\n";
      break;
    default:
      if (V == kVec)
        o << "  *(float4*)((float*)out + i0) = make_float4(" << r << "[0], " << r << "[1], "
          << r << "[2], " << r << "[3]);\n  *(float4*)((float*)out + i0 + 4) = make_float4("
          << r << "[4], " << r << "[5], " << r << "[6], " << r << "[7]);\n";
      else
        o << "  ((float*)out)[i0] = " << r << "[0];\n";
  }
  o << "}\n";
  return o.str();
}

struct Entry {
  std::string cubin;
  std::unordered_map<int, cudaKernel_t> kernels;  // device -> loaded kernel
  std::vector<cudaLibrary_t> libs;
};

std::mutex g_mu;
std::unordered_map<std::string, std::unique_ptr<Entry>>& cache() {
  static auto* c = new std::unordered_map<std::string, std::unique_ptr<Entry>>();
  return *c;  // never destroyed: libraries stay loaded until the process exits
}

// Compile (or find) the kernel for `key`; returns nullptr with the error set.
Entry* compiled(const std::string& key, const kvm_ew_program& p, const Shape& s) {
  auto it = cache().find(key);
  if (it != cache().end()) return it->second.get();
  const Nvrtc* n = nvrtc();
  if (!n) return nullptr;
  const std::string src = source_of(p, s);
  nvrtcProgram prog = nullptr;
  nvrtcResult r = n->Create(&prog, src.c_str(), "kvm_ew.cu", 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) {
    fail(KVM_ERR_CUDA, std::string("nvrtcCreateProgram: ") + n->ErrorString(r));
    return nullptr;
  }
  // --fmad=false: every instruction rounds on its own, as in the interpreter
  // (a multiply feeding an add is not contracted into one FMA).
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "--fmad=false"};
  r = n->Compile(prog, 3, opts);
  if (r != NVRTC_SUCCESS) {
    size_t len = 0;
    n->LogSize(prog, &len);
    std::string log(len, '\0');
    if (len) n->Log(prog, log.data());
    n->Destroy(&prog);
    fail(KVM_ERR_CUDA, "elementwise codegen: NVRTC failed: " + log);
    return nullptr;
  }
  auto e = std::make_unique<Entry>();
  size_t len = 0;
  n->CubinSize(prog, &len);
  e->cubin.resize(len);
  n->Cubin(prog, e->cubin.data());
  n->Destroy(&prog);
  Entry* raw = e.get();
  cache()[key] = std::move(e);
  return raw;
}

}  // namespace

bool ew_jit_enabled() {
  const char* e = std::getenv("KVM_SM100_EW_JIT");  // read per call: A/B in one process
  return !(e && e[0] == '0');
}

int ew_jit_prepare(const kvm_ew_program& p, const kvm_ew_inputs& in, const void* out,
                   int64_t n) {
  const Shape s = choose(p, in, out, n);
  std::lock_guard<std::mutex> lock(g_mu);
  return compiled(key_of(p, s), p, s) ? KVM_OK : KVM_ERR_CUDA;
}

int ew_jit_launch(const kvm_ew_program& p, const kvm_ew_inputs& in, void* out, int64_t n,
                  cudaStream_t stream) {
  const Shape s = choose(p, in, out, n);
  cudaKernel_t kern = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    Entry* e = compiled(key_of(p, s), p, s);
    if (!e) return KVM_ERR_CUDA;
    int dev = 0;
    KVM_CUDA_TRY(cudaGetDevice(&dev));
    auto k = e->kernels.find(dev);
    if (k == e->kernels.end()) {
      cudaLibrary_t lib = nullptr;
      KVM_CUDA_TRY(cudaLibraryLoadData(&lib, e->cubin.data(), nullptr, nullptr, 0, nullptr,
                                       nullptr, 0));
      e->libs.push_back(lib);
      KVM_CUDA_TRY(cudaLibraryGetKernel(&kern, lib, "kvm_ew"));
      e->kernels[dev] = kern;
    } else {
      kern = k->second;
    }
  }
  const uint64_t nvec = uint64_t(n) / uint64_t(s.vec);
  const uint64_t blocks = (nvec + kThreads - 1) / kThreads;
  if (blocks > 0x7FFFFFFFull) return fail(KVM_ERR_INVALID_ARG, "elementwise: n too large");
  void* args[KVM_EW_MAX_INPUTS + 2];
  const void* ptrs[KVM_EW_MAX_INPUTS];
  for (int i = 0; i < p.n_inputs; ++i) {
    ptrs[i] = in.ptr[i];
    args[i] = &ptrs[i];
  }
  void* o = out;
  uint64_t nv = nvec;
  args[p.n_inputs] = &o;
  args[p.n_inputs + 1] = &nv;
  KVM_CUDA_TRY(cudaLaunchKernel(reinterpret_cast<const void*>(kern),
                                dim3(unsigned(blocks)), dim3(kThreads), args, 0, stream));
  return KVM_OK;
}

}  // namespace kvm
