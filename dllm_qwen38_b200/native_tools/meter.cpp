// meter: bounded block-diffusion decode with per-call and per-phase accounting.
//
//   meter --model <preset|hf-dir> --prompt prompt.json --blocks N --out DIR
//         [--block 32] [--threshold 0.9] [--sub-block 0] [--eos ID] [--num-layers N]
//
// prompt.json holds one {"ids": [...]} object. Contract (the reference's llama.cpp meter,
// `tools/weight-space/meter.cpp:171-291`, re-targeted at this framework's cached block decoder):
//   * fixed decoding rule: temperature 0, confidence threshold, optional sub-block window;
//   * every engine call is timed on the host (the engine synchronizes the device before it returns)
//     and accounted to its phase (prefill / decode) with the block passes it ran;
//   * a call that runs a different number of block passes than declared (prefill: one per whole
//     prompt block; step: one; commit: one) fails the run ("undeclared graph visits");
//   * outputs: DIR/tokens.txt (generated ids), DIR/calls.jsonl (one line per call),
//     DIR/meter.json (per-phase and overall counts and times).
#include <sys/stat.h>

#include <chrono>
#include <fstream>
#include <sstream>

#include "embed.hpp"

using namespace bdllm_tools;

namespace {
struct Phase {
  long calls = 0, passes = 0;
  double wall_ms = 0;
};

long passes_of(PyObject* session) {
  PyObject* p = PyObject_GetAttrString(session, "passes");
  check(p, "session.passes");
  long v = PyLong_AsLong(p);
  Py_DECREF(p);
  return v;
}
}  // namespace

int main(int argc, char** argv) {
  std::string model, prompt_path, out, root;
  int blocks = 0, block = 32, sub_block = 0, num_layers = 0;
  long eos = -1;
  double threshold = 0.9;
  for (int i = 1; i < argc; ++i) {
    std::string a = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) die("missing value for " + a);
      return argv[++i];
    };
    if (a == "--model") model = next();
    else if (a == "--prompt") prompt_path = next();
    else if (a == "--blocks") blocks = std::atoi(next().c_str());
    else if (a == "--out") out = next();
    else if (a == "--block") block = std::atoi(next().c_str());
    else if (a == "--threshold") threshold = std::atof(next().c_str());
    else if (a == "--sub-block") sub_block = std::atoi(next().c_str());
    else if (a == "--eos") eos = std::atol(next().c_str());
    else if (a == "--num-layers") num_layers = std::atoi(next().c_str());
    else if (a == "--root") root = next();
    else die("unknown argument " + a);
  }
  if (model.empty() || prompt_path.empty() || out.empty() || blocks <= 0 || blocks > 4096 || block <= 0)
    die("usage: meter --model M --prompt P.json --blocks N --out DIR");
  mkdir(out.c_str(), 0755);
  std::vector<long> prompt;
  {
    std::ifstream f(prompt_path);
    if (!f) die("cannot open " + prompt_path);
    std::stringstream ss;
    ss << f.rdbuf();
    prompt = parse_id_array(ss.str(), "ids");
    if (prompt.empty() || prompt.size() > 65536) die("prompt must have 1..65536 tokens");
  }
  if (root.empty()) {
    const char* r = std::getenv("BDLLM_ROOT");
    root = r ? r : ".";
  }
  start_python(root);
  PyObject* m = api();
  PyObject* mdl = PyObject_CallMethod(m, "load", "si", model.c_str(), num_layers);
  check(mdl, "load");
  PyObject* cls = PyObject_GetAttrString(m, "Session");
  check(cls, "Session");
  const long max_len = (long)prompt.size() + (long)(blocks + 1) * block;
  PyObject* sess = PyObject_CallFunction(cls, "Oidil", mdl, block, threshold, sub_block, max_len);
  check(sess, "Session()");
  Phase pre, dec;
  std::ofstream calls(out + "/calls.jsonl");
  auto timed = [&](Phase& ph, const char* phase, const char* api_name, long declared, PyObject* ret_args) {
    const long before = passes_of(sess);
    auto t0 = std::chrono::steady_clock::now();
    PyObject* r = ret_args ? PyObject_CallMethod(sess, api_name, "O", ret_args) : PyObject_CallMethod(sess, api_name, nullptr);
    auto t1 = std::chrono::steady_clock::now();
    check(r, api_name);
    const long ran = passes_of(sess) - before;
    const double ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
    ph.calls += 1;
    ph.passes += ran;
    ph.wall_ms += ms;
    calls << "{\"phase\": \"" << phase << "\", \"call\": \"" << api_name << "\", \"passes\": " << ran
          << ", \"wall_ms\": " << ms << "}\n";
    if (declared >= 0 && ran != declared) {
      calls.flush();
      die(std::string("undeclared block passes in ") + api_name + ": declared " + std::to_string(declared) +
          ", ran " + std::to_string(ran));
    }
    return r;
  };
  PyObject* ids = ids_list(prompt);
  PyObject* r = timed(pre, "prefill", "prefill", (long)(prompt.size() / block), ids);
  Py_DECREF(r);
  Py_DECREF(ids);
  std::vector<long> generated;
  bool stop = false;
  for (int b = 0; b < blocks && !stop; ++b) {
    r = timed(dec, "decode", "begin_block", 0, nullptr);
    long left = PyLong_AsLong(r);
    Py_DECREF(r);
    while (left > 0) {
      r = timed(dec, "decode", "step", 1, nullptr);
      left = PyLong_AsLong(r);
      Py_DECREF(r);
    }
    r = timed(dec, "decode", "commit", 1, nullptr);
    for (long t : to_ids(r)) {
      generated.push_back(t);
      if (t == eos) stop = true;
    }
    Py_DECREF(r);
  }
  calls.close();
  {
    std::ofstream t(out + "/tokens.txt");
    for (long v : generated) t << v << "\n";
  }
  const double total_ms = pre.wall_ms + dec.wall_ms;
  const long total_passes = pre.passes + dec.passes;
  std::ofstream j(out + "/meter.json");
  j << "{\"model\": \"" << json_escape(model) << "\", \"prompt_tokens\": " << prompt.size()
    << ", \"generated\": " << generated.size() << ", \"block\": " << block << ", \"threshold\": " << threshold
    << ", \"sub_block\": " << sub_block << ",\n \"prefill\": {\"calls\": " << pre.calls << ", \"passes\": " << pre.passes
    << ", \"wall_ms\": " << pre.wall_ms << "},\n \"decode\": {\"calls\": " << dec.calls << ", \"passes\": " << dec.passes
    << ", \"wall_ms\": " << dec.wall_ms << "},\n \"total\": {\"calls\": " << (pre.calls + dec.calls)
    << ", \"passes\": " << total_passes << ", \"wall_ms\": " << total_ms << "},\n \"decode_tok_s\": "
    << (dec.wall_ms > 0 ? 1000.0 * generated.size() / dec.wall_ms : 0.0) << ", \"stopped_at_eos\": "
    << (stop ? "true" : "false") << "}\n";
  j.close();
  std::printf("meter: %zu tokens, %ld passes, %.1f ms (decode %.1f ms)\n", generated.size(), total_passes, total_ms,
              dec.wall_ms);
  Py_DECREF(sess);
  Py_DECREF(cls);
  Py_DECREF(mdl);
  Py_FinalizeEx();
  return 0;
}
