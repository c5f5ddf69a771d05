// ref_cg_synth.cu -- hashes of the CG bench's synthetic SPD matrices as the
// reference builds them.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles the reference's own
// bench source (structural/src/bench_cg_solve.cu, named by REF_BENCH, read
// where it lies) into this translation unit with its main() renamed, so the
// file-static generators make_synthetic_spd (:205-238) and
// make_synthetic_laplacian_spd (:245-278) are called directly; nothing of
// that source is copied.  tests/golden/make_cg_synth_golden.py runs the
// result (oracle/_ref/ref_cg_synth) and writes tests/golden/cg_synth.json.
//
// usage: ref_cg_synth synth|lapl N HALFBW SEED PARAM
// prints: nnz, then FNV-1a 64 of row_ptr (as int64), col_idx (as int32) and
// values (as IEEE double bytes), little-endian.
#define main cove_reference_bench_main
#include REF_BENCH
#undef main

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace {

struct Fnv {
    std::uint64_t h = 1469598103934665603ULL;
    void bytes(const void* p, std::size_t n) {
        const auto* c = static_cast<const unsigned char*>(p);
        for (std::size_t i = 0; i < n; ++i) h = (h ^ c[i]) * 1099511628211ULL;
    }
};

}  // namespace

int main(int argc, char** argv) {
    if (argc != 6) {
        std::fprintf(stderr, "usage: %s synth|lapl N HALFBW SEED PARAM\n", argv[0]);
        return 2;
    }
    const int n = std::atoi(argv[2]), bw = std::atoi(argv[3]);
    const unsigned seed = static_cast<unsigned>(std::strtoul(argv[4], nullptr, 10));
    const double param = std::strtod(argv[5], nullptr);
    const auto a = std::strcmp(argv[1], "lapl") == 0 ? make_synthetic_laplacian_spd(n, bw, seed, param)
                                                     : make_synthetic_spd(n, bw, seed, param);
    Fnv rp, ci, va;
    for (const auto p : a.row_ptr) {
        const std::int64_t v = p;
        rp.bytes(&v, 8);
    }
    for (const auto c : a.col_idx) {
        const std::int32_t v = c;
        ci.bytes(&v, 4);
    }
    for (const double v : a.values) va.bytes(&v, 8);
    std::printf("nnz %lld\nrow_ptr %016llx\ncol_idx %016llx\nvalues %016llx\n",
                static_cast<long long>(a.row_ptr.back()), static_cast<unsigned long long>(rp.h),
                static_cast<unsigned long long>(ci.h), static_cast<unsigned long long>(va.h));
    return 0;
}
