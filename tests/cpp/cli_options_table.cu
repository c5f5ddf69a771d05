// Runs the family CLI's option handling (spmv_cli_options.hpp) on cases
// read from stdin, through the public structural:: API only, so the same
// source builds against the reference's headers (oracle/Makefile ->
// oracle/_ref/ref_cli_options; tests/golden/make_cli_options_golden.py
// stores its answers) and against this library's shim
// (tests/test_cli_options.py), and the answers must be equal.
//
// Input lines:
//   N layout|codec|policy|alg SPELLING   normalised name (layouts also the algorithm)
//   K layout|codec|policy NAME           enum value of a normalised name
//   P MATRIX [ARGS...]                   parse_spmv_cli_options on the argument list
#include "structural/spmv_cli_options.hpp"

#include <cstdio>
#include <exception>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

using namespace structural;

int main() {
    std::string line;
    while (std::getline(std::cin, line)) {
        std::istringstream in(line);
        std::string op;
        in >> op;
        std::cout << line << " => ";
        try {
            if (op == "N") {
                std::string kind, s;
                in >> kind >> s;
                if (kind == "layout") {
                    std::string alg = "keep";
                    const std::string l = normalize_spmv_layout_name(s, alg);
                    std::cout << l << " " << alg;
                } else if (kind == "codec") {
                    std::cout << normalize_spmv_value_codec_name(s);
                } else if (kind == "policy") {
                    std::cout << normalize_spmv_load_balance_policy_name(s);
                } else {
                    std::cout << normalize_cusparse_spmv_alg_name(s);
                }
            } else if (op == "K") {
                std::string kind, s;
                in >> kind >> s;
                if (kind == "layout") std::cout << static_cast<int>(spmv_layout_kind_from_name(s));
                else if (kind == "codec") std::cout << static_cast<int>(spmv_value_codec_kind_from_name(s));
                else std::cout << static_cast<int>(spmv_load_balance_policy_from_name(s));
            } else {
                std::vector<std::string> args{"struct_gpu_spmv"};
                for (std::string a; in >> a;) args.push_back(a);
                std::vector<char*> argv;
                for (auto& a : args) argv.push_back(&a[0]);
                const auto o = parse_spmv_cli_options(static_cast<int>(argv.size()), argv.data());
                std::cout << o.matrix_path << " " << o.precision << " " << o.layout << " " << o.value_codec << " "
                          << o.lb_chunk_blocks << " " << o.lb_split_threshold_blocks << " " << o.lb_policy << " "
                          << o.lb_chunk_blocks_explicit << o.lb_split_threshold_blocks_explicit << " "
                          << spmv_has_manual_load_balance_override(o) << " " << o.cusparse_alg << " " << o.warmup
                          << " " << o.iterations << " " << o.verify_cpu;
            }
        } catch (const std::exception& e) {
            std::cout << "ERR " << e.what();
        }
        std::cout << "\n";
    }
    return 0;
}
