// blob_fuzz_test.cpp -- test infrastructure: feeds reef's packed model blob
// reader (reef_b200/csrc/blob.cpp) valid and corrupted blobs on the CPU, built
// with AddressSanitizer.  A blob comes from a file the caller may not control,
// so every malformed one must end in an error status, never a read outside
// the blob or a write outside the arena.  The device copies are host copies
// here (fake_cuda_nccl.cpp), so ASan sees every byte the loader touches; the
// weight repacking kernel is a no-op stand-in.
//
// Usage: blob_fuzz_test <blob file>...  For each blob: the unmodified blob
// must load (every layer of a W8A8 blob, and the whole model); then seeded
// mutations -- header fields and layer-table fields set to boundary and
// random values, truncations, byte flips -- each go through read_info and,
// when that accepts them, the layer and model loads.  Prints
// "ok <file> <mutations> <accepted>" per blob; exits non-zero on a failure.
#include "ops.h"
#include "reef_b200.h"

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace reef {

int check_device() { return kOk; }
int pack_weight_i8(long long, long long, const int8_t*, int8_t*, long long, cudaStream_t) {
  return kOk;
}

}  // namespace reef

namespace {

constexpr size_t kCap = size_t{256} << 20;  // larger arenas are not allocated here
constexpr int kMaxLayers = 64;

struct Rng {
  uint64_t s;
  uint32_t next() {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return static_cast<uint32_t>(s >> 33);
  }
};

// Loads what the blob's header admits; returns the number of calls that
// returned OK.
int exercise(const std::vector<uint8_t>& b) {
  reef_b200_blob_info info{};
  if (reef_b200_blob_read_info(b.data(), b.size(), &info) != REEF_B200_OK) return 0;
  int ok = 1;
  const size_t lb = reef_b200_blob_layer_bytes(&info);
  if (info.precision == 1 && lb > 0 && lb <= kCap) {
    void* arena = std::aligned_alloc(256, (lb + 255) / 256 * 256);
    const size_t layers = info.layers < 8 ? info.layers : 8;
    for (size_t l = 0; l < layers + 1; ++l) {  // one past the last: refused
      reef_b200_gptneo_block blk{};
      if (reef_b200_blob_load_layer(b.data(), b.size(), l, arena, lb, &blk, nullptr) ==
          REEF_B200_OK)
        ++ok;
    }
    std::free(arena);
  }
  const size_t mb = reef_b200_blob_model_bytes(&info);
  if (mb > 0 && mb <= kCap && info.layers <= kMaxLayers) {
    void* arena = std::aligned_alloc(256, (mb + 255) / 256 * 256);
    std::vector<reef_b200_gptneo_block> blocks(info.layers);
    std::vector<reef_b200_gptneo_block_f32> blocks_f32(info.layers);
    reef_b200_gptneo_model model{};
    if (reef_b200_blob_load_model(b.data(), b.size(), arena, mb, &model, blocks.data(),
                                  blocks_f32.data(), nullptr) == REEF_B200_OK)
      ++ok;
    std::free(arena);
  }
  return ok;
}

uint32_t rd32(const std::vector<uint8_t>& b, size_t at) {
  uint32_t v;
  std::memcpy(&v, b.data() + at, 4);
  return v;
}

void wr32(std::vector<uint8_t>& b, size_t at, uint32_t v) { std::memcpy(b.data() + at, &v, 4); }

}  // namespace

int main(int argc, char** argv) {
  int failures = 0;
  for (int a = 1; a < argc; ++a) {
    FILE* f = std::fopen(argv[a], "rb");
    if (f == nullptr) {
      std::fprintf(stderr, "FAIL cannot open %s\n", argv[a]);
      ++failures;
      continue;
    }
    std::vector<uint8_t> blob;
    uint8_t buf[65536];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) blob.insert(blob.end(), buf, buf + n);
    std::fclose(f);

    // the blob as written loads: header, every layer (W8A8), the whole model
    reef_b200_blob_info info{};
    if (reef_b200_blob_read_info(blob.data(), blob.size(), &info) != REEF_B200_OK) {
      std::fprintf(stderr, "FAIL %s: the unmodified blob is refused\n", argv[a]);
      ++failures;
      continue;
    }
    const int want = 1 + (info.precision == 1 ? static_cast<int>(info.layers < 8 ? info.layers : 8)
                                              : 0) +
                     1;
    const int got = exercise(blob);
    if (got != want) {
      std::fprintf(stderr, "FAIL %s: %d of %d loads of the unmodified blob succeeded\n", argv[a],
                   got, want);
      ++failures;
      continue;
    }
    const uint32_t layers_at = rd32(blob, 60);  // Header::layers
    const size_t table = static_cast<size_t>(info.layers) * 80;
    Rng rng{0x5eed0000ull + static_cast<uint64_t>(a)};
    int mutations = 0, accepted = 0;
    for (int it = 0; it < 4000; ++it) {
      std::vector<uint8_t> m = blob;
      const uint32_t size = static_cast<uint32_t>(m.size());
      const uint32_t pick[] = {0u, 1u, 15u, 16u, size - 16u, size, size + 16u, 0x7ffffff0u,
                               0xfffffff0u, 0xffffffffu, rng.next()};
      const uint32_t value = pick[rng.next() % (sizeof pick / sizeof pick[0])];
      switch (rng.next() % 4) {
        case 0:  // a header field
          wr32(m, 4 * (rng.next() % 17), value);
          break;
        case 1:  // a field of a layer record
          if (table > 0 && layers_at + table <= m.size())
            wr32(m, layers_at + 4 * (rng.next() % (table / 4)), value);
          break;
        case 2:  // a shorter blob
          m.resize(rng.next() % (m.size() + 1));
          break;
        default:  // a few flipped bytes in the header and layer table
          for (int k = 0; k < 4; ++k) {
            const size_t span = layers_at + table < m.size() ? layers_at + table : m.size();
            const size_t at = span > 0 ? rng.next() % span : 0;
            if (at < m.size()) m[at] ^= static_cast<uint8_t>(1u << (rng.next() % 8));
          }
      }
      ++mutations;
      // a fresh buffer of exactly the blob's length (a shrunk vector keeps its
      // old capacity), so a read past the end is a read outside the allocation
      const std::vector<uint8_t> view(m.begin(), m.end());
      if (exercise(view) > 0) ++accepted;
    }
    std::printf("ok %s %d %d\n", argv[a], mutations, accepted);
  }
  std::fflush(stdout);
  return failures == 0 ? 0 : 1;
}
