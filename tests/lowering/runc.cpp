// runc.cpp -- gcc-compiled execution of rendered C kernels (TEST
// INFRASTRUCTURE), in the manner of the reference's CpuDevice::compile /
// execute (src/device/cpu.rs:151-208, 318-380): one shared object per source,
// looked up by name and called with one argument per parameter slot.
#include <dlfcn.h>
#include <unistd.h>

#include <cstdlib>
#include <fstream>
#include <functional>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <unordered_map>

#include "lowering.h"

namespace kir {
namespace {

std::string cache_dir() {
  const char *e = std::getenv("FG_LOWERING_CACHE");
  return e && *e ? e : "/tmp/fg_lowering_cache";
}

// "void name(float* restrict data0, int data2) {" -> a trampoline taking
// void** indexed by slot.
std::string trampoline(const std::string &code, const std::string &name) {
  const std::string head = "void " + name + "(";
  size_t p = code.find(head);
  if (p == std::string::npos) throw std::runtime_error("run_c: no function " + name);
  size_t q = code.find(')', p);
  std::string params = code.substr(p + head.size(), q - p - head.size());
  std::ostringstream call;
  call << "\nvoid fg_entry(void **a) {\n  " << name << "(";
  size_t start = 0;
  bool first = true;
  while (start < params.size()) {
    size_t comma = params.find(',', start);
    if (comma == std::string::npos) comma = params.size();
    std::string prm = params.substr(start, comma - start);
    start = comma + 1;
    size_t d = prm.rfind("data");
    if (d == std::string::npos) continue;
    const std::string slot = prm.substr(d + 4);
    std::string type = prm.substr(0, d);
    while (!type.empty() && type.front() == ' ') type.erase(type.begin());
    const bool ptr = type.find('*') != std::string::npos;
    std::string base = type.substr(0, type.find_first_of("* "));
    if (!first) call << ", ";
    first = false;
    if (ptr)
      call << "(" << base << "*)a[" << slot << "]";
    else
      call << "*(" << base << "*)a[" << slot << "]";
  }
  call << ");\n}\n";
  return call.str();
}

using Entry = void (*)(void **);

Entry compile(const std::string &code, const std::string &name) {
  static std::unordered_map<std::string, Entry> programs;
  const char *cf = std::getenv("FG_LOWERING_CFLAGS");
  const std::string src = code + trampoline(code, name) + "// " + (cf ? cf : "") + "\n";
  auto it = programs.find(src);
  if (it != programs.end()) return it->second;
  const std::string dir = cache_dir();
  if (std::system(("mkdir -p " + dir).c_str()) != 0)
    throw std::runtime_error("run_c: cannot create " + dir);
  const std::string stem =
      dir + "/k" + std::to_string(std::hash<std::string>()(src)) + "_" + std::to_string(getpid());
  {
    std::ofstream f(stem + ".c");
    f << src;
  }
  // FG_LOWERING_CFLAGS replaces the optimisation flags (the reference builds
  // with clang -O3 -march=native; -ffp-contract=off stays, so no product is
  // fused into an FMA under any setting)
  const std::string flags = std::string(cf && *cf ? cf : "-O2") + " -ffp-contract=off";
  const std::string cmd = "gcc " + flags + " -fPIC -shared -o " + stem + ".so " + stem +
                          ".c -lm 2> " + stem + ".log";
  if (std::system(cmd.c_str()) != 0) {
    std::ifstream l(stem + ".log");
    std::stringstream m;
    m << l.rdbuf();
    throw std::runtime_error("run_c: gcc failed: " + m.str() + "\n" + src);
  }
  void *h = dlopen((stem + ".so").c_str(), RTLD_NOW | RTLD_LOCAL);
  if (!h) throw std::runtime_error(std::string("run_c: dlopen: ") + dlerror());
  auto fn = reinterpret_cast<Entry>(dlsym(h, "fg_entry"));
  if (!fn) throw std::runtime_error("run_c: no entry point");
  programs.emplace(src, fn);
  return fn;
}

}  // namespace

void run_c(const std::string &code, const std::string &name, const std::vector<void *> &args) {
  Entry fn = compile(code, name);
  std::vector<void *> a = args;
  fn(a.data());
}

}  // namespace kir
