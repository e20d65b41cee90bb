// User `kernel` bodies: MSL (as malus-codegen-gpu emits it) -> CUDA C++ ->
// NVRTC -> sm_100a cubin, launched with the reference's buffer conventions.
//
// The reference's runtime_init receives, per kernel id, the MSL text that
// codegen-gpu produced (crates/malus-codegen-gpu/src/lib.rs:432-1006) and
// compiles it with Metal.  Here the same text is translated to CUDA C++ and
// compiled once per distinct source with NVRTC for sm_100a.  The translated
// subset is exactly what the emitter produces:
//   * implicit-map kernels: `device T* p [[buffer(i)]]` inputs, `out`, and
//     `uint tid [[thread_position_in_grid]]`; body `T x = ...; out[tid] = ...;`
//     (Metal dispatches exactly len threads; CUDA launches whole blocks, so a
//     `tid < n` guard is added);
//   * explicit kernels: `device const T*` inputs, `device T* out`, an optional
//     `constant Uniforms_<id>& u`, one `constant TensorMeta& <t>_meta` per
//     tensor, and the thread-position attributes it uses; bodies with lets,
//     assignments, if/for/while, `threadgroup T a[N]` arrays,
//     `threadgroup_barrier(mem_flags::mem_threadgroup)`, and the float math
//     calls exp/log/sqrt/rsqrt/tanh/fabs/fmax/fmin/pow.
// Buffer slots follow the runtime's binding (metal.rs:1944-2065): inputs
// 0..hc-1, out hc, uniforms hc+1, TensorMeta hc+2.. (inputs, then out).
// Uniforms and TensorMeta are passed by value as kernel parameters.
#include "common.cuh"

#include <cuda.h>
#include <nvrtc.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <regex>
#include <sstream>
#include <string>
#include <vector>

namespace malus {

struct JitParam {
  enum Kind { Ptr, Uniforms, Meta, Attr } kind;
  int buffer = -1;        // Metal buffer slot (Ptr, Uniforms, Meta)
  std::string name;       // parameter / variable name
  std::string attr;       // Attr: the Metal attribute
};

struct JitKernel {
  std::string name, cuda;
  std::vector<JitParam> params;   // Ptr/Uniforms/Meta in signature order
  bool implicit = false;          // `uint tid [[thread_position_in_grid]]` form
  size_t uniform_bytes = 0;       // sizeof(Uniforms_<id>) (4 bytes per field)
  CUfunction fn = nullptr;
};

namespace {

struct TensorMetaHost {
  uint32_t ndim;
  uint32_t shape[8];
  uint32_t strides[8];
};

std::string trim(const std::string& s) {
  size_t a = s.find_first_not_of(" \t\r\n"), b = s.find_last_not_of(" \t\r\n");
  return a == std::string::npos ? std::string() : s.substr(a, b - a + 1);
}

// top-level comma split (the emitted parameter lists hold no nested commas)
std::vector<std::string> split_params(const std::string& s) {
  std::vector<std::string> out;
  int depth = 0;
  std::string cur;
  for (char c : s) {
    if (c == '(' || c == '[') ++depth;
    if (c == ')' || c == ']') --depth;
    if (c == ',' && depth == 0) {
      out.push_back(trim(cur));
      cur.clear();
    } else {
      cur += c;
    }
  }
  if (!trim(cur).empty()) out.push_back(trim(cur));
  return out;
}

const char* attr_expr(const std::string& a) {
  if (a == "thread_position_in_grid") return "(uint)(blockIdx.x * blockDim.x + threadIdx.x)";
  if (a == "threadgroup_position_in_grid") return "(uint)blockIdx.x";
  if (a == "thread_position_in_threadgroup") return "(uint)threadIdx.x";
  if (a == "threads_per_threadgroup") return "(uint)blockDim.x";
  if (a == "threads_per_grid") return "(uint)(gridDim.x * blockDim.x)";
  return nullptr;
}

}  // namespace

// MSL -> CUDA C++; throws std::runtime_error with the reason on unsupported input.
std::string msl_to_cuda(const std::string& msl, JitKernel* k) {
  std::string src = msl;
  src = std::regex_replace(src, std::regex(R"(#include\s*<metal_stdlib>)"), "");
  src = std::regex_replace(src, std::regex(R"(using\s+namespace\s+metal\s*;)"), "");
  std::smatch m;
  if (!std::regex_search(src, m, std::regex(R"(kernel\s+void\s+([A-Za-z_]\w*)\s*\()")))
    throw std::runtime_error("no `kernel void name(` in the source");
  k->name = m[1];
  const size_t sig_start = m.position(0), open = m.position(0) + m.length(0);
  int depth = 1;
  size_t close = open;
  for (; close < src.size() && depth; ++close) {
    if (src[close] == '(') ++depth;
    if (src[close] == ')') --depth;
  }
  if (depth) throw std::runtime_error("unbalanced parameter list");
  const std::string plist = src.substr(open, close - 1 - open);
  const size_t body_open = src.find('{', close);
  const size_t body_close = src.rfind('}');
  if (body_open == std::string::npos || body_close == std::string::npos || body_close < body_open)
    throw std::runtime_error("kernel body not found");
  std::string body = src.substr(body_open + 1, body_close - body_open - 1);
  const std::string prefix = src.substr(0, sig_start);   // struct definitions

  std::vector<std::string> cparams, locals;
  const std::regex re_ptr(R"(^device\s+(const\s+)?(\w+)\s*\*\s*(\w+)\s*\[\[\s*buffer\((\d+)\)\s*\]\]$)");
  const std::regex re_uni(R"(^constant\s+(\w+)\s*&\s*(\w+)\s*\[\[\s*buffer\((\d+)\)\s*\]\]$)");
  const std::regex re_attr(R"(^uint\s+(\w+)\s*\[\[\s*(\w+)\s*\]\]$)");
  for (const std::string& p : split_params(plist)) {
    std::smatch pm;
    if (std::regex_match(p, pm, re_ptr)) {
      JitParam q{JitParam::Ptr, std::stoi(pm[4]), pm[3], ""};
      k->params.push_back(q);
      cparams.push_back((pm[1].matched ? "const " : "") + pm[2].str() + "* __restrict__ " + pm[3].str());
    } else if (std::regex_match(p, pm, re_uni)) {
      const std::string ty = pm[1], nm = pm[2];
      JitParam q{ty == "TensorMeta" ? JitParam::Meta : JitParam::Uniforms, std::stoi(pm[3]), nm, ""};
      k->params.push_back(q);
      cparams.push_back("const " + ty + " " + nm);
    } else if (std::regex_match(p, pm, re_attr)) {
      const char* e = attr_expr(pm[2]);
      if (!e) throw std::runtime_error("unsupported thread attribute " + pm[2].str());
      locals.push_back("const uint " + pm[1].str() + " = " + e + ";");
      if (pm[1] == "tid" && pm[2] == "thread_position_in_grid") k->implicit = true;
    } else {
      throw std::runtime_error("unsupported kernel parameter: " + p);
    }
  }
  // Uniforms struct size: 4 bytes per field (the runtime packs them so)
  for (const JitParam& q : k->params) {
    if (q.kind != JitParam::Uniforms) continue;
    std::smatch sm;
    const std::regex re_struct("struct\\s+" + std::string("Uniforms_\\w+") + "\\s*\\{([^}]*)\\}");
    if (std::regex_search(prefix, sm, re_struct)) {
      std::string fields = sm[1];
      k->uniform_bytes = 4 * (size_t)std::count(fields.begin(), fields.end(), ';');
    }
  }
  cparams.push_back("const unsigned long long __malus_n");
  // body: barriers, shared arrays, float math
  body = std::regex_replace(body, std::regex(R"(threadgroup_barrier\s*\(\s*mem_flags::mem_threadgroup\s*\))"),
                            "__syncthreads()");
  body = std::regex_replace(body, std::regex(R"(\bthreadgroup\s+)"), "__shared__ ");
  static const char* fmap[][2] = {{"exp", "expf"},   {"log", "logf"},   {"sqrt", "sqrtf"},
                                  {"rsqrt", "rsqrtf"}, {"tanh", "tanhf"}, {"fabs", "fabsf"},
                                  {"fmax", "fmaxf"}, {"fmin", "fminf"}, {"pow", "powf"}};
  for (auto& f : fmap)
    body = std::regex_replace(body, std::regex(std::string("\\b") + f[0] + "\\s*\\("), std::string(f[1]) + "(");
  body = std::regex_replace(body, std::regex(R"(\bNaNf\b)"), "__int_as_float(0x7fffffff)");
  body = std::regex_replace(body, std::regex(R"(-inff\b)"), "__int_as_float(0xff800000)");
  body = std::regex_replace(body, std::regex(R"(\binff\b)"), "__int_as_float(0x7f800000)");
  if (std::regex_search(body, std::regex(R"(\b(simd_\w+|atomic_\w+|texture\w*|sampler)\b)")))
    throw std::runtime_error("unsupported Metal construct in kernel body");

  std::ostringstream o;
  o << "typedef unsigned int uint;\ntypedef unsigned short ushort;\ntypedef unsigned char uchar;\n"
       "typedef unsigned long long ulong;\n";
  if (src.find("half") != std::string::npos) o << "#include <cuda_fp16.h>\ntypedef __half half;\n";
  o << prefix << "\nextern \"C\" __global__ void " << k->name << "(";
  for (size_t i = 0; i < cparams.size(); ++i) o << (i ? ", " : "") << cparams[i];
  o << ") {\n";
  for (const std::string& l : locals) o << "  " << l << "\n";
  if (k->implicit) o << "  if ((unsigned long long)tid >= __malus_n) return;\n";
  o << body << "\n}\n";
  return o.str();
}

namespace {

using PFN_load = CUresult (*)(CUmodule*, const void*);
using PFN_getf = CUresult (*)(CUfunction*, CUmodule, const char*);
using PFN_launch = CUresult (*)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                                unsigned, CUstream, void**, void**);
PFN_load g_load = nullptr;
PFN_getf g_getf = nullptr;
PFN_launch g_launch = nullptr;

void load_driver() {
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* f = nullptr;
    MALUS_CUDA(cudaGetDriverEntryPointByVersion("cuModuleLoadData", &f, 12000, cudaEnableDefault, &q));
    g_load = (PFN_load)f;
    MALUS_CUDA(cudaGetDriverEntryPointByVersion("cuModuleGetFunction", &f, 12000, cudaEnableDefault, &q));
    g_getf = (PFN_getf)f;
    MALUS_CUDA(cudaGetDriverEntryPointByVersion("cuLaunchKernel", &f, 12000, cudaEnableDefault, &q));
    g_launch = (PFN_launch)f;
    if (!g_load || !g_getf || !g_launch) panic("CUDA driver entry points for module loading unavailable");
  });
}

// NVRTC: CUDA C++ -> sm_100a cubin.  Returns "" and fills *log on failure.
std::string nvrtc_cubin(const std::string& cuda, const std::string& name, std::string* log) {
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, cuda.c_str(), (name + ".cu").c_str(), 0, nullptr, nullptr) != NVRTC_SUCCESS) {
    *log = "nvrtcCreateProgram failed";
    return "";
  }
  const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "--fmad=false",
                        "-I/usr/local/cuda/include"};
  nvrtcResult r = nvrtcCompileProgram(prog, 4, opts);
  size_t ls = 0;
  nvrtcGetProgramLogSize(prog, &ls);
  std::string lg(ls, '\0');
  if (ls) nvrtcGetProgramLog(prog, &lg[0]);
  std::string cubin;
  if (r == NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetCUBINSize(prog, &n);
    cubin.resize(n);
    nvrtcGetCUBIN(prog, &cubin[0]);
  } else {
    *log = lg;
  }
  nvrtcDestroyProgram(&prog);
  return cubin;
}

std::mutex g_jit_mu;
std::map<std::string, JitKernel*> g_jit_cache;   // by MSL source text

}  // namespace

bool looks_like_msl(const char* s) { return s && std::strstr(s, "kernel void") != nullptr; }

JitKernel* jit_compile(const std::string& msl) {
  std::lock_guard<std::mutex> lk(g_jit_mu);
  auto it = g_jit_cache.find(msl);
  if (it != g_jit_cache.end()) return it->second;
  auto* k = new JitKernel();
  try {
    k->cuda = msl_to_cuda(msl, k);
  } catch (const std::exception& e) {
    panic("runtime_init: cannot translate kernel source: %s", e.what());
  }
  std::string log;
  std::string cubin = nvrtc_cubin(k->cuda, k->name, &log);
  if (cubin.empty()) panic("runtime_init: NVRTC failed for %s:\n%s", k->name.c_str(), log.c_str());
  load_driver();
  stream();   // bind the device / primary context
  CUmodule mod;
  if (g_load(&mod, cubin.data()) != CUDA_SUCCESS) panic("runtime_init: loading %s failed", k->name.c_str());
  if (g_getf(&k->fn, mod, k->name.c_str()) != CUDA_SUCCESS)
    panic("runtime_init: %s not found in its module", k->name.c_str());
  g_jit_cache[msl] = k;
  return k;
}

namespace {

TensorMetaHost meta_of(int64_t h) {
  TensorMetaHost t{};
  auto* b = tb(h);
  t.ndim = (uint32_t)b->ndim;
  size_t st = 1;
  for (int d = b->ndim - 1; d >= 0; --d) {
    t.shape[d] = (uint32_t)b->shape[d];
    t.strides[d] = (uint32_t)st;
    st *= b->shape[d];
  }
  return t;
}

void jit_launch(JitKernel* k, const int64_t* h, size_t hc, int64_t out, const void* u, size_t ub,
                unsigned gx, unsigned gy, unsigned gz, unsigned bx, unsigned by, unsigned bz,
                unsigned long long n) {
  std::vector<void*> ptrs(k->params.size());
  std::vector<TensorMetaHost> metas(k->params.size());
  std::vector<unsigned char> uni(std::max<size_t>(k->uniform_bytes, 4), 0);
  std::vector<void*> args;
  for (size_t i = 0; i < k->params.size(); ++i) {
    const JitParam& q = k->params[i];
    if (q.kind == JitParam::Ptr) {
      if ((size_t)q.buffer < hc) ptrs[i] = vptr(h[q.buffer]);
      else if ((size_t)q.buffer == hc) ptrs[i] = vptr(out);
      else panic("kernel %s: buffer(%d) is not an input or the output", k->name.c_str(), q.buffer);
      args.push_back(&ptrs[i]);
    } else if (q.kind == JitParam::Uniforms) {
      if (ub < k->uniform_bytes) panic("kernel %s: %zu uniform bytes, %zu needed", k->name.c_str(), ub, k->uniform_bytes);
      if (k->uniform_bytes) memcpy(uni.data(), u, k->uniform_bytes);
      args.push_back(uni.data());
    } else {   // Meta: slots hc+2.. = inputs, then out
      size_t t = (size_t)q.buffer - (hc + 2);
      if (q.buffer < (int)hc + 2 || t > hc) panic("kernel %s: TensorMeta slot %d out of range", k->name.c_str(), q.buffer);
      metas[i] = meta_of(t < hc ? h[t] : out);
      args.push_back(&metas[i]);
    }
  }
  args.push_back(&n);
  CUresult r = g_launch(k->fn, gx, gy, gz, bx, by, bz, 0, (CUstream)stream(), args.data(), nullptr);
  if (r != CUDA_SUCCESS) panic("launch of %s failed (%d)", k->name.c_str(), (int)r);
  count_launch();
  after_launch(k->name.c_str());
}

}  // namespace

// kernel_dispatch: exactly len(inputs[0]) threads (Metal dispatchThreads).
void jit_dispatch_implicit(JitKernel* k, const int64_t* h, size_t count, int64_t out) {
  size_t n = tb(out)->len;
  if (!n) return;
  jit_launch(k, h, count, out, nullptr, 0, (unsigned)((n + 255) / 256), 1, 1, 256, 1, 1, n);
}

// kernel_dispatch_v2: grid = threadgroups, tg = threads per threadgroup
// (Metal dispatchThreadgroups).
void jit_dispatch_explicit(JitKernel* k, const int64_t* h, size_t hc, const size_t* grid, const size_t* tg,
                           int64_t out, const void* u, size_t ub) {
  if (tg[0] * tg[1] * tg[2] > 1024) panic("kernel %s: threadgroup of %zu threads", k->name.c_str(), tg[0] * tg[1] * tg[2]);
  if (!grid[0] || !grid[1] || !grid[2]) return;
  jit_launch(k, h, hc, out, u, ub, (unsigned)grid[0], (unsigned)grid[1], (unsigned)grid[2], (unsigned)tg[0],
             (unsigned)tg[1], (unsigned)tg[2], ~0ull);
}

}  // namespace malus

using namespace malus;

extern "C" int32_t malus_jit_translate(const char* msl, char* out, size_t cap) {
  JitKernel k;
  std::string s;
  try {
    s = msl_to_cuda(msl ? msl : "", &k);
  } catch (const std::exception& e) {
    s = std::string("error: ") + e.what();
    if (out && cap) snprintf(out, cap, "%s", s.c_str());
    return -1;
  }
  if (out && cap) snprintf(out, cap, "%s", s.c_str());
  return (int32_t)s.size();
}

extern "C" int32_t malus_jit_compile_check(const char* msl, char* log, size_t cap) {
  JitKernel k;
  std::string cuda;
  try {
    cuda = msl_to_cuda(msl ? msl : "", &k);
  } catch (const std::exception& e) {
    if (log && cap) snprintf(log, cap, "translate: %s", e.what());
    return -1;
  }
  std::string lg;
  std::string cubin = nvrtc_cubin(cuda, k.name, &lg);
  if (log && cap) snprintf(log, cap, "%s", lg.c_str());
  return cubin.empty() ? -2 : 0;
}
