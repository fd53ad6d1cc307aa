// Host f32 -> f16 cast of the C++ API (funasr_b200::f32_to_f16_bits), run over a file of
// f32 values; writes the f16 bit patterns for the test to compare with numpy's cast.
#include "funasr_b200.hpp"

#include <cstdio>
#include <vector>

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    FILE* in = std::fopen(argv[1], "rb");
    if (!in) return 2;
    std::vector<float> x;
    float f;
    while (std::fread(&f, 4, 1, in) == 1) x.push_back(f);
    std::fclose(in);
    std::vector<uint16_t> y(x.size());
    for (size_t i = 0; i < x.size(); ++i) y[i] = funasr_b200::f32_to_f16_bits(x[i]);
    FILE* out = std::fopen(argv[2], "wb");
    if (!out) return 2;
    std::fwrite(y.data(), 2, y.size(), out);
    std::fclose(out);
    return 0;
}
