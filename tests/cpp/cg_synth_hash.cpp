// Hashes of structural::make_synthetic_spd / make_synthetic_laplacian_spd
// (cove-spmv_b200/include/structural/synthetic_spd.hpp) in the format of
// oracle/ref_cg_synth.cu, for tests/test_cg_bench_cli.py to compare with
// the reference generators' hashes in tests/golden/cg_synth.json.
#include "structural/synthetic_spd.hpp"

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
    const auto a = std::strcmp(argv[1], "lapl") == 0 ? structural::make_synthetic_laplacian_spd(n, bw, seed, param)
                                                     : structural::make_synthetic_spd(n, bw, seed, param);
    a.validate();
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
