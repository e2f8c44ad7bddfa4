// shifts.cpp -- the random-shift offsets of the separators (TEST INFRASTRUCTURE ONLY).
//
// src/htdemucs.cpp:578, 617-619 and src/roformer.cpp:461-465 draw each shift's offset with
// std::mt19937 and std::uniform_int_distribution<int>; the distribution's algorithm belongs to
// the standard library, so the checker draws through the same library calls.
#include <random>

extern "C" int or_shift_offsets(unsigned seed, int shifts, int hi, int* out) {
    if (shifts < 0 || hi < 0 || (shifts > 0 && !out)) return -1;
    std::mt19937 rng(seed);
    std::uniform_int_distribution<int> dist(0, hi);
    for (int k = 0; k < shifts; k++) out[k] = dist(rng);
    return 0;
}
