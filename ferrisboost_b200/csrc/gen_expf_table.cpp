// Build step: list every f32 input on which the host C library's expf differs
// from fexp_core (fexp.h), with the host's result.  Evaluates both functions on
// all 2^32 bit patterns (OpenMP) and writes a sorted binary table:
//   "FBEXPT01" | u64 count | count x (u32 input bits, u32 expf bits)
// Usage: gen_expf_table <out.bin>
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <utility>
#include <vector>

#include <omp.h>

#include "fexp.h"

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <out.bin>\n", argv[0]);
        return 2;
    }
    const int nth = omp_get_max_threads();
    std::vector<std::vector<std::pair<uint32_t, uint32_t>>> part(nth);
#pragma omp parallel
    {
        auto& mine = part[omp_get_thread_num()];
#pragma omp for schedule(dynamic, 1 << 20)
        for (long long u = 0; u < (1ll << 32); u++) {
            const uint32_t key = (uint32_t)u;
            float x;
            std::memcpy(&x, &key, 4);
            const float g = expf(x);
            const float m = fbx::fexp_core(x);
            uint32_t gb, mb;
            std::memcpy(&gb, &g, 4);
            std::memcpy(&mb, &m, 4);
            if (gb != mb && !(std::isnan(g) && std::isnan(m))) mine.push_back({key, gb});
        }
    }
    std::vector<std::pair<uint32_t, uint32_t>> all;
    for (auto& p : part) all.insert(all.end(), p.begin(), p.end());
    std::sort(all.begin(), all.end());
    FILE* f = std::fopen(argv[1], "wb");
    if (!f) return 1;
    const char magic[8] = {'F', 'B', 'E', 'X', 'P', 'T', '0', '1'};
    const uint64_t n = all.size();
    std::fwrite(magic, 1, 8, f);
    std::fwrite(&n, 8, 1, f);
    for (auto& e : all) {
        std::fwrite(&e.first, 4, 1, f);
        std::fwrite(&e.second, 4, 1, f);
    }
    std::fclose(f);
    std::printf("%llu exceptions\n", (unsigned long long)n);
    return 0;
}
