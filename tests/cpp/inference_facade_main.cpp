// Drives the chess_engine_4::inference facade the way the lc0 ce4 backend does:
//   inference_facade_main <model.safetensors> <planes.bin> <batch> <out.bin>
// planes.bin holds batch * 112 InputPlane records (16 bytes each); out.bin receives
// policy [batch, policy_size], wdl [batch, 3], moves_left [batch] as float32.
#include <chess_engine_4/inference.h>

#include <cstdio>
#include <exception>
#include <fstream>
#include <vector>

int main(int argc, char** argv) {
  using namespace chess_engine_4::inference;
  if (argc != 5) {
    std::fprintf(stderr, "usage: %s model planes batch out\n", argv[0]);
    return 2;
  }
  try {
    const int batch = std::atoi(argv[3]);
    auto model = Model::Load(argv[1], 0, batch);
    std::vector<InputPlane> planes(static_cast<size_t>(batch) * 112);
    std::ifstream in(argv[2], std::ios::binary);
    for (auto& p : planes) {
      std::uint64_t raw[2];
      in.read(reinterpret_cast<char*>(raw), sizeof(raw));
      p.mask = raw[0];
      p.value = *reinterpret_cast<const float*>(&raw[1]);
    }
    if (!in) throw std::runtime_error("short planes file");
    const int ps = model->info().policy_size;
    std::vector<float> policy(static_cast<size_t>(batch) * ps), wdl(batch * 3), ml(batch);
    model->Evaluate(planes, batch, {.policy = policy, .wdl = wdl, .moves_left = ml});
    // A span that is too small must throw, as the reference engine's checks do.
    bool threw = false;
    try {
      model->Evaluate(planes, batch, {.policy = std::span<float>(policy).first(1), .wdl = wdl, .moves_left = ml});
    } catch (const std::runtime_error&) {
      threw = true;
    }
    if (!threw) throw std::runtime_error("undersized output span was accepted");
    std::ofstream out(argv[4], std::ios::binary);
    out.write(reinterpret_cast<const char*>(policy.data()), policy.size() * 4);
    out.write(reinterpret_cast<const char*>(wdl.data()), wdl.size() * 4);
    out.write(reinterpret_cast<const char*>(ml.data()), ml.size() * 4);
    std::printf("ok d_model=%d depth=%d policy_size=%d\n", model->info().d_model, model->info().depth, ps);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "error: %s\n", e.what());
    return 1;
  }
}
