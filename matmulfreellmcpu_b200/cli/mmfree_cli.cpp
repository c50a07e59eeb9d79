// mmfree_cli.cpp -- drop-in for the reference's mmfree-cli (matmulfreellmCPU cpp/app/main.cpp)
// running on one B200 through libmmfree_cuda.so.
//
// Same flags and output: a text prompt (the positional argument, else stdin) or --ids a,b,c,
// --blob --tokenizer (default <blob dir>/tokenizer.mmtok) --mode float|fixed (default fixed)
// --frac --gen --temp --top-k --seed --decode-ids a,b,c --no-bos --no-eos --print-ids
// --show-ids --logits-out PATH --bench --warmup --reps, plus --device N.
//   text mode  the prompt is tokenized (tokenizer.hpp), generation stops at </s> (unless
//              --no-eos) and the new tokens are decoded and streamed to stdout as they are
//              produced, then a newline (main.cpp:186-215); --print-ids prints the id stream
//   --ids mode the full id stream (prompt + generated) is printed space-separated and there
//              is no EOS stop (main.cpp:134-145, 211, 236-240)
//   --decode-ids decodes ids to text without a model; --gen 0 --print-ids tokenizes only.
// --logits-out writes the last-position logits of the full stream as raw float32
// (main.cpp:217-224). --profile is not supported (device time is measured with CUDA events).
#include <cctype>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <iostream>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "mmfree_cuda.hpp"
#include "tokenizer.hpp"

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

// tokenizer.mmtok beside the weight blob (main.cpp:77-81)
std::string default_tokenizer(const std::string& blob) {
  const std::size_t slash = blob.find_last_of('/');
  return (slash == std::string::npos ? std::string() : blob.substr(0, slash + 1)) + "tokenizer.mmtok";
}

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
  std::string blob = "model.mmfree", mode = "fixed", ids_arg, logits_out, tok_path, prompt,
              decode_arg;
  bool print_ids = false, show_ids = false, bench = false, have_seed = false, have_prompt = false,
       no_bos = false, no_eos = false;
  int frac = 10, warmup = 1, reps = 3, device = 0;
  std::size_t gen = 32;
  mmfree::cuda::Sampling samp;
  for (int a = 1; a < argc; ++a) {
    std::string k = argv[a];
    auto next = [&]() { return (a + 1 < argc) ? argv[++a] : ""; };
    if (k == "--blob") blob = next();
    else if (k == "--tokenizer") tok_path = next();
    else if (k == "--mode") mode = next();
    else if (k == "--frac") frac = std::atoi(next());
    else if (k == "--gen") gen = static_cast<std::size_t>(std::atoll(next()));
    else if (k == "--temp" || k == "--temperature") samp.temperature = static_cast<float>(std::atof(next()));
    else if (k == "--top-k") samp.top_k = std::atoi(next());
    else if (k == "--seed") { samp.seed = std::strtoull(next(), nullptr, 10); have_seed = true; }
    else if (k == "--ids") ids_arg = next();
    else if (k == "--decode-ids") decode_arg = next();
    else if (k == "--no-bos") no_bos = true;
    else if (k == "--no-eos") no_eos = true;
    else if (k == "--print-ids") print_ids = true;
    else if (k == "--show-ids") show_ids = true;
    else if (k == "--logits-out") logits_out = next();
    else if (k == "--bench") bench = true;
    else if (k == "--warmup") warmup = std::atoi(next());
    else if (k == "--reps") reps = std::atoi(next());
    else if (k == "--device") device = std::atoi(next());
    else if (k == "--profile") {
      std::fprintf(stderr, "--profile: not supported (time the device with CUDA events)\n");
      return 2;
    } else if (!k.empty() && k[0] == '-') {
      std::fprintf(stderr, "unknown arg: %s\n", k.c_str());
      return 2;
    } else {
      prompt = k;  // a positional argument is the prompt text
      have_prompt = true;
    }
  }
  if (tok_path.empty()) tok_path = default_tokenizer(blob);
  std::unique_ptr<mmfree_cli::Tokenizer> tok;
  try {
    if (!decode_arg.empty()) {  // tokenizer only, no model
      mmfree_cli::Tokenizer t(tok_path);
      std::printf("%s\n", t.decode(parse_ids(decode_arg)).c_str());
      return 0;
    }
    const bool ids_mode = !ids_arg.empty();
    const bool ids_out = print_ids || ids_mode;
    if (!ids_mode || !ids_out) tok = std::make_unique<mmfree_cli::Tokenizer>(tok_path);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  const bool ids_mode = !ids_arg.empty();
  const bool ids_out = print_ids || ids_mode;
  std::vector<std::int64_t> ids;
  if (ids_mode) {
    ids = parse_ids(ids_arg);
  } else {
    if (!have_prompt) {
      if (bench) {
        prompt = "The quick brown fox jumps over the lazy dog.";
      } else {  // the prompt from stdin, trailing newlines and spaces removed
        std::string all, line;
        while (std::getline(std::cin, line)) all += line + "\n";
        while (!all.empty() && (all.back() == '\n' || all.back() == ' ')) all.pop_back();
        prompt = all;
      }
    }
    ids = tok->encode(prompt, !no_bos);
  }
  if (ids.empty()) {
    std::fprintf(stderr, "no input (pass a prompt, --ids, or pipe via stdin)\n");
    return 2;
  }
  const ActQuant aq = mode == "fixed" ? ActQuant::FixedQ510 : ActQuant::Float;
  if (!(gen > 0 || !logits_out.empty() || bench)) {  // tokenization only: no model
    if (show_ids) {
      std::fprintf(stderr, "prompt ids (%zu):", ids.size());
      for (auto t : ids) std::fprintf(stderr, " %lld", static_cast<long long>(t));
      std::fprintf(stderr, "\ngen ids (0):\n");
    }
    if (ids_out) {
      for (std::size_t i = 0; i < ids.size(); ++i)
        std::printf("%lld%s", static_cast<long long>(ids[i]), i + 1 < ids.size() ? " " : "\n");
    } else {
      std::printf("%s\n", tok->decode({}).c_str());
    }
    return 0;
  }
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
    // text out: re-decode the generated ids at every token and print the new bytes (BPE
    // decode is prefix-stable, so the stream is byte-identical to decoding at the end)
    std::vector<std::int64_t> shown_ids;
    std::string shown;
    std::function<void(std::int64_t)> on_token;
    if (!ids_out) {
      on_token = [&](std::int64_t id) {
        shown_ids.push_back(id);
        std::string full = tok->decode(shown_ids);
        if (full.size() > shown.size()) {
          std::fwrite(full.data() + shown.size(), 1, full.size() - shown.size(), stdout);
          std::fflush(stdout);
        }
        shown = std::move(full);
      };
    }
    const std::int64_t eos = (!ids_mode && !no_eos && tok) ? tok->eos_id() : -1;
    std::vector<std::int64_t> stream = gen > 0 ? model.generate(ids, gen, eos, samp, on_token) : ids;
    if (!ids_out && gen > 0) std::fputc('\n', stdout);
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
    if (ids_out) {
      for (std::size_t i = 0; i < stream.size(); ++i)
        std::printf("%lld%s", static_cast<long long>(stream[i]), i + 1 < stream.size() ? " " : "\n");
    } else if (gen == 0) {
      std::printf("%s\n", tok->decode({}).c_str());
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
  return 0;
}
