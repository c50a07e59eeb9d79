// seam_check.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Runs the UNMODIFIED reference engine (matmulfreellmCPU Model, linked from oracle/_ref objects
// built from its own sources) twice on one blob in FixedQ510 mode: once with its default
// CpuBackend, once with mmfree::cuda::CudaTernaryBackend (include/mmfree_cuda_backend.hpp)
// injected through Model::set_backend (model.hpp:74-79). Compares, bit for bit:
//   - Model::forward logits of a prompt (prefill rows reach the backend in batches),
//   - Model::generate ids (hgrn_model.cpp:249-347, batch-1 decode),
//   - Model::generate_serve ids (hgrn_model.cpp:349-454, lockstep batches of B rows),
// and prints one line per check; exit status 0 only if every check matches.
//
//   seam_check BLOB [batch]
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "mmfree/model.hpp"
#include "mmfree/weights.hpp"
#include "mmfree_cuda_backend.hpp"

namespace {

std::vector<std::int64_t> ids_from(std::uint64_t seed, std::size_t n, std::size_t vocab) {
  std::vector<std::int64_t> v(n);
  std::uint64_t s = seed * 6364136223846793005ull + 1442695040888963407ull;
  for (auto& t : v) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    t = 3 + static_cast<std::int64_t>((s >> 33) % (vocab - 3));
  }
  return v;
}

int report(const char* what, bool ok) {
  std::printf("%s %s\n", what, ok ? "match" : "DIFFER");
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: seam_check BLOB [batch]\n");
    return 2;
  }
  const std::size_t batch = argc > 2 ? std::strtoul(argv[2], nullptr, 10) : 256;
  try {
    mmfree::Weights w(argv[1]);
    const std::size_t V = w.config().vocab_size;
    mmfree::Model cpu(w, mmfree::ActQuant::FixedQ510, 10);
    mmfree::Model gpu(w, mmfree::ActQuant::FixedQ510, 10);
    mmfree::cuda::CudaTernaryBackend be(0, batch);
    gpu.set_backend(&be, {});

    int bad = 0;
    const auto prompt = ids_from(1, 37, V);
    std::vector<float> lc, lg;
    cpu.forward(prompt.data(), prompt.size(), lc);
    gpu.forward(prompt.data(), prompt.size(), lg);
    bad += report("forward_logits",
                  lc.size() == lg.size() && std::memcmp(lc.data(), lg.data(), 4 * lc.size()) == 0);

    const auto a = cpu.generate(prompt, 12);
    const auto b = gpu.generate(prompt, 12);
    bad += report("generate_ids", a == b);

    std::vector<std::vector<std::int64_t>> prompts = {ids_from(2, 5, V), ids_from(3, 9, V),
                                                      ids_from(4, 9, V), ids_from(5, 1, V)};
    const auto sa = cpu.generate_serve(prompts, 7);
    const auto sb = gpu.generate_serve(prompts, 7);
    bad += report("generate_serve_ids", sa == sb);

    std::printf("ids:");
    for (auto t : b) std::printf(" %lld", static_cast<long long>(t));
    std::printf("\n");
    return bad ? 1 : 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "seam_check: %s\n", e.what());
    return 3;
  }
}
