// Embedded-interpreter plumbing shared by the native tools (capture, meter).
//
// The tools are C++ programs that own argument parsing, limits, file formats, timing and
// accounting, and drive this framework's engine through `dllm_qwen38_b200.native_tools.api`
// inside an embedded CPython. The interpreter is the one named by BDLLM_PYTHON (default: the
// `python3` found on PATH), so its virtual environment's packages (torch) are visible; the
// repository root is put on sys.path.
#pragma once
#include <Python.h>

#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace bdllm_tools {

[[noreturn]] inline void die(const std::string& msg) {
  std::fprintf(stderr, "error: %s\n", msg.c_str());
  std::exit(1);
}

inline std::string which(const char* exe) {
  const char* path = std::getenv("PATH");
  if (!path) return exe;
  std::string p(path);
  size_t s = 0;
  while (s <= p.size()) {
    size_t e = p.find(':', s);
    if (e == std::string::npos) e = p.size();
    std::string cand = p.substr(s, e - s) + "/" + exe;
    if (FILE* f = std::fopen(cand.c_str(), "rb")) {
      std::fclose(f);
      return cand;
    }
    s = e + 1;
  }
  return exe;
}

// Start the interpreter; `root` is prepended to sys.path.
inline void start_python(const std::string& root) {
  PyConfig cfg;
  PyConfig_InitPythonConfig(&cfg);
  const char* env = std::getenv("BDLLM_PYTHON");
  std::string exe = env ? env : which("python3");
  PyStatus st = PyConfig_SetBytesString(&cfg, &cfg.program_name, exe.c_str());
  if (PyStatus_Exception(st)) die("python config");
  st = PyConfig_SetBytesString(&cfg, &cfg.executable, exe.c_str());
  if (PyStatus_Exception(st)) die("python config");
  cfg.install_signal_handlers = 0;
  st = Py_InitializeFromConfig(&cfg);
  PyConfig_Clear(&cfg);
  if (PyStatus_Exception(st)) die("cannot start the embedded interpreter");
  PyObject* sys_path = PySys_GetObject("path");  // borrowed
  PyObject* r = PyUnicode_FromString(root.c_str());
  PyList_Insert(sys_path, 0, r);
  Py_DECREF(r);
}

inline void check(PyObject* o, const char* what) {
  if (o == nullptr) {
    PyErr_Print();
    die(std::string("python call failed: ") + what);
  }
}

inline PyObject* api() {
  static PyObject* m = nullptr;
  if (!m) {
    m = PyImport_ImportModule("dllm_qwen38_b200.native_tools.api");
    check(m, "import dllm_qwen38_b200.native_tools.api");
  }
  return m;
}

inline PyObject* ids_list(const std::vector<long>& ids) {
  PyObject* l = PyList_New((Py_ssize_t)ids.size());
  for (size_t i = 0; i < ids.size(); ++i) PyList_SET_ITEM(l, (Py_ssize_t)i, PyLong_FromLong(ids[i]));
  return l;
}

inline std::vector<long> to_ids(PyObject* l) {
  std::vector<long> out;
  PyObject* seq = PySequence_Fast(l, "expected a sequence of ints");
  check(seq, "sequence");
  const Py_ssize_t n = PySequence_Fast_GET_SIZE(seq);
  for (Py_ssize_t i = 0; i < n; ++i) out.push_back(PyLong_AsLong(PySequence_Fast_GET_ITEM(seq, i)));
  Py_DECREF(seq);
  return out;
}

// "[1, 2, 3]" -> ids (the JSON arrays of the prompt files; no other JSON is parsed)
inline std::vector<long> parse_id_array(const std::string& line, const char* key) {
  std::vector<long> out;
  size_t k = line.find(std::string("\"") + key + "\"");
  if (k == std::string::npos) die(std::string("line without \"") + key + "\": " + line.substr(0, 80));
  size_t a = line.find('[', k), b = line.find(']', a == std::string::npos ? k : a);
  if (a == std::string::npos || b == std::string::npos) die("malformed id array");
  std::string body = line.substr(a + 1, b - a - 1);
  size_t s = 0;
  while (s < body.size()) {
    while (s < body.size() && (body[s] == ' ' || body[s] == ',' || body[s] == '\n')) ++s;
    if (s >= body.size()) break;
    char* end = nullptr;
    long v = std::strtol(body.c_str() + s, &end, 10);
    if (end == body.c_str() + s) die("non-integer token id");
    out.push_back(v);
    s = (size_t)(end - body.c_str());
  }
  return out;
}

inline std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') o += '\\', o += c;
    else if (c == '\n') o += "\\n";
    else if ((unsigned char)c < 0x20) {
      char b[8];
      std::snprintf(b, sizeof b, "\\u%04x", c);
      o += b;
    } else o += c;
  }
  return o;
}

}  // namespace bdllm_tools
