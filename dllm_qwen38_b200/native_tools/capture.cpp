// capture: dump the residual stream after chosen layers for a few prompts.
//
//   capture --model <preset|hf-dir> --prompts prompts.jsonl --layers 31,35,39 --out DIR
//           [--block 32] [--num-layers N]
//
// prompts.jsonl holds one {"ids": [...]} object per line. Contract (the reference's llama.cpp
// capture tool, `tools/weight-space/capture.cpp:27-151`, re-targeted at this framework's engine):
//   * at most 8 prompts, each line at most 64 KiB and at most 4096 tokens; anything else is rejected
//     before the model is loaded;
//   * one forward per prompt; every captured tensor must be float32, C-contiguous, 2-D [T, D] and at
//     most 64 MiB, else the run fails;
//   * files DIR/p<j>-l<layer>.f32 (raw little-endian float32, row-major) with one JSONL line per file
//     in DIR/index.jsonl: {"prompt", "layer", "file", "rows", "cols", "bytes"};
//   * DIR/status.json: {"ok", "prompts", "tensors", "layer_visits", "error"} written on every exit
//     path that gets past argument parsing.
#include <sys/stat.h>

#include <cstring>
#include <fstream>
#include <sstream>

#include "embed.hpp"

using namespace bdllm_tools;

namespace {
constexpr int kMaxPrompts = 8;
constexpr size_t kMaxLine = 64 * 1024;
constexpr size_t kMaxTokens = 4096;
constexpr size_t kMaxTensorBytes = 64ull << 20;

std::string g_out;

void write_status(bool ok, int prompts, int tensors, long visits, const std::string& err) {
  std::ofstream f(g_out + "/status.json");
  f << "{\"ok\": " << (ok ? "true" : "false") << ", \"prompts\": " << prompts << ", \"tensors\": " << tensors
    << ", \"layer_visits\": " << visits << ", \"error\": \"" << json_escape(err) << "\"}\n";
}

[[noreturn]] void fail(const std::string& msg, int prompts, int tensors, long visits) {
  write_status(false, prompts, tensors, visits, msg);
  die(msg);
}
}  // namespace

int main(int argc, char** argv) {
  std::string model, prompts_path, layers_s, root;
  int block = 32, num_layers = 0;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) die("missing value for " + a);
      return argv[++i];
    };
    if (a == "--model") model = next();
    else if (a == "--prompts") prompts_path = next();
    else if (a == "--layers") layers_s = next();
    else if (a == "--out") g_out = next();
    else if (a == "--block") block = std::atoi(next().c_str());
    else if (a == "--num-layers") num_layers = std::atoi(next().c_str());
    else if (a == "--root") root = next();
    else die("unknown argument " + a);
  }
  if (model.empty() || prompts_path.empty() || layers_s.empty() || g_out.empty())
    die("usage: capture --model M --prompts P.jsonl --layers a,b --out DIR");
  mkdir(g_out.c_str(), 0755);
  std::vector<int> layers;
  {
    std::stringstream ss(layers_s);
    std::string t;
    while (std::getline(ss, t, ',')) layers.push_back(std::atoi(t.c_str()));
  }
  // read and validate every prompt before touching the model
  std::vector<std::vector<long>> prompts;
  {
    std::ifstream f(prompts_path);
    if (!f) fail("cannot open " + prompts_path, 0, 0, 0);
    std::string line;
    while (std::getline(f, line)) {
      if (line.find_first_not_of(" \t\r") == std::string::npos) continue;
      if (line.size() > kMaxLine) fail("prompt line longer than 64 KiB", 0, 0, 0);
      if ((int)prompts.size() == kMaxPrompts) fail("more than 8 prompts", 0, 0, 0);
      auto ids = parse_id_array(line, "ids");
      if (ids.empty() || ids.size() > kMaxTokens) fail("prompt must have 1..4096 tokens", 0, 0, 0);
      prompts.push_back(std::move(ids));
    }
  }
  if (prompts.empty()) fail("no prompts", 0, 0, 0);
  if (root.empty()) {
    const char* r = std::getenv("BDLLM_ROOT");
    root = r ? r : ".";
  }
  start_python(root);
  PyObject* m = api();
  PyObject* mdl = PyObject_CallMethod(m, "load", "si", model.c_str(), num_layers);
  if (!mdl) {
    PyErr_Print();
    fail("model load failed", 0, 0, 0);
  }
  PyObject* layer_list = PyList_New((Py_ssize_t)layers.size());
  for (size_t i = 0; i < layers.size(); ++i) PyList_SET_ITEM(layer_list, (Py_ssize_t)i, PyLong_FromLong(layers[i]));
  std::ofstream index(g_out + "/index.jsonl");
  int tensors = 0;
  long visits = 0;
  for (size_t j = 0; j < prompts.size(); ++j) {
    PyObject* ids = ids_list(prompts[j]);
    PyObject* res = PyObject_CallMethod(m, "capture", "OOOi", mdl, ids, layer_list, block);
    Py_DECREF(ids);
    if (!res) {
      PyErr_Print();
      fail("capture call failed", (int)j, tensors, visits);
    }
    PyObject* dict = PyTuple_GetItem(res, 0);  // borrowed
    visits += PyLong_AsLong(PyTuple_GetItem(res, 1));
    for (int layer : layers) {
      PyObject* key = PyLong_FromLong(layer);
      PyObject* arr = PyDict_GetItemWithError(dict, key);  // borrowed
      Py_DECREF(key);
      if (!arr) fail("layer " + std::to_string(layer) + " not captured", (int)j, tensors, visits);
      Py_buffer view;
      if (PyObject_GetBuffer(arr, &view, PyBUF_C_CONTIGUOUS | PyBUF_FORMAT | PyBUF_ND) != 0) {
        PyErr_Clear();
        fail("captured tensor is not a C-contiguous buffer", (int)j, tensors, visits);
      }
      const bool f32 = view.format && std::strcmp(view.format, "f") == 0 && view.itemsize == 4;
      if (!f32 || view.ndim != 2) {
        PyBuffer_Release(&view);
        fail("captured tensor is not 2-D float32", (int)j, tensors, visits);
      }
      if ((size_t)view.len > kMaxTensorBytes) {
        PyBuffer_Release(&view);
        fail("captured tensor larger than 64 MiB", (int)j, tensors, visits);
      }
      const std::string name = "p" + std::to_string(j) + "-l" + std::to_string(layer) + ".f32";
      {
        std::ofstream out(g_out + "/" + name, std::ios::binary);
        out.write(reinterpret_cast<const char*>(view.buf), view.len);
        if (!out) {
          PyBuffer_Release(&view);
          fail("write failed: " + name, (int)j, tensors, visits);
        }
      }
      index << "{\"prompt\": " << j << ", \"layer\": " << layer << ", \"file\": \"" << name
            << "\", \"rows\": " << view.shape[0] << ", \"cols\": " << view.shape[1] << ", \"bytes\": " << view.len
            << "}\n";
      PyBuffer_Release(&view);
      ++tensors;
    }
    Py_DECREF(res);
  }
  index.close();
  write_status(true, (int)prompts.size(), tensors, visits, "");
  std::printf("capture: %zu prompts, %d tensors, %ld layer visits -> %s\n", prompts.size(), tensors, visits,
              g_out.c_str());
  Py_DECREF(layer_list);
  Py_DECREF(mdl);
  Py_FinalizeEx();
  return 0;
}
