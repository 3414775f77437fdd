// TEST INFRASTRUCTURE ONLY. Driver linked against the reference's own
// core/src/ssim.cpp (createSSIMWindow, ssim.cpp:7-24), compiled from the
// reference sources by oracle/Makefile (target ref) into oracle/_ref/. Prints
// the 11x11 window the reference builds, one float per line as an exact
// hexadecimal float, for tests/golden/make_ref_constants.py.
#include <cstdio>
#include <vector>

std::vector<float> createSSIMWindow(int windowSize, float sigma);

int main() {
    const std::vector<float> w = createSSIMWindow(11, 1.5f);
    for (float v : w) std::printf("%a\n", (double)v);
    return 0;
}
