// mmfree_cli.cpp -- drop-in for the reference's mmfree-cli raw-ids path (matmulfreellmCPU
// cpp/app/main.cpp) running on one B200 through libmmfree_cuda.so.
//
// Same flags and output: --blob --mode float|fixed (default fixed) --frac --gen --temp --top-k
// --seed --ids a,b,c --print-ids --show-ids --logits-out PATH --bench --warmup --reps, plus
// --device N. In --ids mode the full id stream (prompt + generated) is printed space-separated
// on stdout and there is no EOS stop, as in main.cpp:134-145,211,236-240. --logits-out writes
// the last-position logits of the full stream as raw float32 (main.cpp:217-224). Text prompts
// need the reference's tokenizer, which this build does not include: they are rejected.
#include <cctype>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "mmfree_cuda.hpp"

using mmfree::cuda::ActQuant;

namespace {

std::vector<std::int64_t> parse_ids(const std::string& s) {  // main.cpp:62-75
  std::vector<std::int64_t> ids;
  std::size_t i = 0;
  while (i < s.size()) {
    while (i < s.size() && !(std::isdigit(static_cast<unsigned char>(s[i])) || s[i] == '-')) ++i;
    if (i >= s.size()) break;
    std::size_t j = i;
    if (s[j] == '-') ++j;
    while (j < s.size() && std::isdigit(static_cast<unsigned char>(s[j]))) ++j;
    ids.push_back(std::stoll(s.substr(i, j - i)));
    i = j;
  }
  return ids;
}

using clk = std::chrono::steady_clock;
double secs(clk::duration d) { return std::chrono::duration<double>(d).count(); }

// Timing with the split of the reference's run_bench (bench.cpp:51-66): prefill ends with the
// first generated token, decode covers the remaining gen-1 tokens.
int run_bench(mmfree::cuda::Model& m, const std::vector<std::int64_t>& ids, std::size_t gen,
              int warmup, int reps, const std::string& blob, const std::string& mode, int frac) {
  auto once = [&](double& pre, double& dec) {
    const std::int64_t* p = ids.data();
    std::size_t n = ids.size();
    std::int64_t first = 0;
    auto t0 = clk::now();
    mmfree::cuda::check(mmfree_cuda_serve_begin(m.handle(), 1, &p, &n, &first));
    auto t1 = clk::now();
    std::vector<std::int64_t> rest(gen > 1 ? gen - 1 : 0);
    if (gen > 1) mmfree::cuda::check(mmfree_cuda_serve_run(m.handle(), gen - 1, rest.data()));
    auto t2 = clk::now();
    mmfree::cuda::check(mmfree_cuda_serve_end(m.handle()));
    pre = secs(t1 - t0);
    dec = secs(t2 - t1);
  };
  std::printf("mmfree-cli benchmark (CUDA)\n");
  std::printf("  blob:          %s\n", blob.c_str());
  std::printf("  mode:          %s (frac=%d)\n", mode.c_str(), frac);
  std::printf("  device:        B200 (sm_100a)\n");
  std::printf("  prompt tokens: %zu\n", ids.size());
  std::printf("  gen tokens:    %zu\n", gen);
  std::printf("  warmup/reps:   %d/%d\n\n", warmup, reps);
  double pre = 0, dec = 0;
  for (int i = 0; i < warmup; ++i) once(pre, dec);
  double sum_pre = 0, sum_tps = 0, sum_total = 0;
  for (int i = 0; i < reps; ++i) {
    once(pre, dec);
    const double tps = (gen > 1 && dec > 0) ? (gen - 1) / dec : 0.0;
    const double total = pre + dec;
    std::printf("  run %d: prefill %7.1f ms   decode %8.2f tok/s   overall %8.2f tok/s\n", i + 1,
                pre * 1e3, tps, total > 0 ? gen / total : 0.0);
    sum_pre += pre;
    sum_tps += tps;
    sum_total += total;
  }
  const double n = reps > 0 ? reps : 1;
  std::printf("\n  avg prefill: %7.1f ms  (%.2f tok/s over %zu prompt tokens)\n", sum_pre / n * 1e3,
              sum_pre > 0 ? ids.size() / (sum_pre / n) : 0.0, ids.size());
  std::printf("  avg decode:  %8.2f tok/s\n", sum_tps / n);
  std::printf("  avg overall: %8.2f tok/s  (%zu gen tokens / %.3f s)\n",
              sum_total > 0 ? gen / (sum_total / n) : 0.0, gen, sum_total / n);
  return 0;
}

}  // namespace

int main(int argc, char** argv) {
  std::string blob = "model.mmfree", mode = "fixed", ids_arg, logits_out;
  bool print_ids = false, show_ids = false, bench = false, have_seed = false;
  int frac = 10, warmup = 1, reps = 3, device = 0;
  std::size_t gen = 32;
  mmfree::cuda::Sampling samp;
  for (int a = 1; a < argc; ++a) {
    std::string k = argv[a];
    auto next = [&]() { return (a + 1 < argc) ? argv[++a] : ""; };
    if (k == "--blob") blob = next();
    else if (k == "--mode") mode = next();
    else if (k == "--frac") frac = std::atoi(next());
    else if (k == "--gen") gen = static_cast<std::size_t>(std::atoll(next()));
    else if (k == "--temp" || k == "--temperature") samp.temperature = static_cast<float>(std::atof(next()));
    else if (k == "--top-k") samp.top_k = std::atoi(next());
    else if (k == "--seed") { samp.seed = std::strtoull(next(), nullptr, 10); have_seed = true; }
    else if (k == "--ids") ids_arg = next();
    else if (k == "--print-ids") print_ids = true;
    else if (k == "--show-ids") show_ids = true;
    else if (k == "--logits-out") logits_out = next();
    else if (k == "--bench") bench = true;
    else if (k == "--warmup") warmup = std::atoi(next());
    else if (k == "--reps") reps = std::atoi(next());
    else if (k == "--device") device = std::atoi(next());
    else if (k == "--tokenizer" || k == "--decode-ids" || k == "--no-bos" || k == "--no-eos" ||
             k == "--profile" || (!k.empty() && k[0] != '-')) {
      std::fprintf(stderr, "%s: text mode needs the reference tokenizer (use --ids)\n", k.c_str());
      return 2;
    } else {
      std::fprintf(stderr, "unknown arg: %s\n", k.c_str());
      return 2;
    }
  }
  (void)print_ids;
  std::vector<std::int64_t> ids = parse_ids(ids_arg);
  if (ids.empty()) {
    std::fprintf(stderr, "no input (pass a prompt, --ids, or pipe via stdin)\n");
    return 2;
  }
  const ActQuant aq = mode == "fixed" ? ActQuant::FixedQ510 : ActQuant::Float;
  try {
    mmfree::cuda::Model model(blob, aq, frac, device);
    if (bench) {
      if (gen == 0) {
        std::fprintf(stderr, "--bench needs --gen > 0\n");
        return 2;
      }
      return run_bench(model, ids, gen, warmup, reps, blob, mode, frac);
    }
    if (samp.temperature > 0.0f && !have_seed) samp.seed = std::random_device{}();
    std::vector<std::int64_t> stream = gen > 0 ? model.generate(ids, gen, -1, samp) : ids;
    if (!logits_out.empty()) {
      std::vector<float> last(model.config().vocab_size);
      mmfree::cuda::check(mmfree_cuda_forward_last(model.handle(), stream.data(), stream.size(),
                                                   last.data()));
      std::ofstream f(logits_out, std::ios::binary);
      f.write(reinterpret_cast<const char*>(last.data()),
              static_cast<std::streamsize>(last.size() * sizeof(float)));
    }
    if (show_ids) {
      std::fprintf(stderr, "prompt ids (%zu):", ids.size());
      for (auto t : ids) std::fprintf(stderr, " %lld", static_cast<long long>(t));
      std::fprintf(stderr, "\ngen ids (%zu):", stream.size() - ids.size());
      for (std::size_t i = ids.size(); i < stream.size(); ++i)
        std::fprintf(stderr, " %lld", static_cast<long long>(stream[i]));
      std::fprintf(stderr, "\n");
    }
    for (std::size_t i = 0; i < stream.size(); ++i)
      std::printf("%lld%s", static_cast<long long>(stream[i]), i + 1 < stream.size() ? " " : "\n");
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  return 0;
}
