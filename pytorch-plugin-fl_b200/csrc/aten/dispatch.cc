// Backend table of the flagos device: backends.conf + FLAGOS_OP_* overrides.
#include "dispatch.h"

#include <dlfcn.h>

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <mutex>
#include <unordered_map>

namespace flb200::aten {
namespace {

std::string Trim(const std::string& s) {
  const size_t l = s.find_first_not_of(" \t\r\n");
  if (l == std::string::npos) return "";
  const size_t r = s.find_last_not_of(" \t\r\n");
  return s.substr(l, r - l + 1);
}

// Parses a backend name; kCount if unknown.
Backend Parse(const std::string& v) {
  if (v == "b200") return Backend::kB200;
  if (v == "cuda") return Backend::kCuda;
  if (v == "flagos" || v == "flaggems") return Backend::kFlagOs;
  if (v == "flagos_python" || v == "flaggems_python") return Backend::kFlagOsPython;
  if (v == "ascend") return Backend::kAscend;
  if (v == "musa") return Backend::kMusa;
  return Backend::kCount;
}

// The package directory holds both _C*.so and backends.conf.
std::string DefaultPath() {
  Dl_info info;
  if (dladdr(reinterpret_cast<void*>(&DefaultPath), &info) && info.dli_fname) {
    std::string lib(info.dli_fname);
    const size_t slash = lib.rfind('/');
    if (slash != std::string::npos) {
      const std::string dir = lib.substr(0, slash);
      for (const char* rel : {"/backends.conf", "/../backends.conf"}) {
        std::ifstream f(dir + rel);
        if (f.is_open()) return dir + rel;
      }
    }
  }
  return "";
}

struct Table {
  std::unordered_map<std::string, Backend> routes;
  std::string path;
};

const Table& GetTable() {
  static const Table table = [] {
    Table t;
    const char* env = std::getenv("FLAGOS_BACKEND_CONFIG");
    t.path = env ? std::string(env) : DefaultPath();
    std::ifstream f(t.path);
    if (!t.path.empty() && f.is_open()) {
      std::string line;
      while (std::getline(f, line)) {
        const size_t hash = line.find('#');
        if (hash != std::string::npos) line.resize(hash);
        const size_t eq = line.find('=');
        if (eq == std::string::npos) continue;
        const std::string op = Trim(line.substr(0, eq));
        const std::string val = Trim(line.substr(eq + 1));
        if (op.empty() || val.empty()) continue;
        const Backend b = Parse(val);
        if (b == Backend::kCount) {
          std::fprintf(stderr, "[flagos] unknown backend '%s' for op '%s' in %s; ignored\n",
                       val.c_str(), op.c_str(), t.path.c_str());
          continue;
        }
        t.routes[op] = b;
      }
    } else {
      t.path.clear();
    }
    return t;
  }();
  return table;
}

}  // namespace

const char* BackendName(Backend b) {
  switch (b) {
    case Backend::kCuda: return "cuda";
    case Backend::kFlagOs: return "flagos";
    case Backend::kFlagOsPython: return "flagos_python";
    case Backend::kAscend: return "ascend";
    case Backend::kMusa: return "musa";
    case Backend::kB200: return "b200";
    default: return "unknown";
  }
}

Backend ConfiguredBackend(const std::string& op) {
  // FLAGOS_OP_<op>, with '.' written as "__" (mm.out -> FLAGOS_OP_mm__out).
  std::string key = "FLAGOS_OP_";
  for (char c : op) {
    if (c == '.') key += "__";
    else key += c;
  }
  if (const char* v = std::getenv(key.c_str())) {
    const Backend b = Parse(Trim(v));
    if (b != Backend::kCount) {
      std::fprintf(stderr, "[flagos] env override: %s -> %s\n", op.c_str(), BackendName(b));
      return b;
    }
    std::fprintf(stderr, "[flagos] unknown backend '%s' in %s; ignored\n", v, key.c_str());
  }
  const auto& routes = GetTable().routes;
  auto it = routes.find(op);
  return it == routes.end() ? Backend::kCount : it->second;
}

bool LogDispatchEnabled() {
  static const bool on = [] {
    const char* v = std::getenv("FLAGOS_LOG_DISPATCH");
    return v && std::string(v) == "1";
  }();
  return on;
}

void LogDispatch(const char* op, Backend b) {
  std::fprintf(stderr, "[flagos dispatch] %s -> %s\n", op, BackendName(b));
}

std::string ConfigPath() { return GetTable().path; }

}  // namespace flb200::aten
