// TEST INFRASTRUCTURE ONLY -- drives the reference's own cache-plan code.
//
// Built by oracle/Makefile from the reference's src/h4 sources where they lie
// (never copied). Two modes, text on stdin/stdout:
//   quotas: "Q n_layers curve_len floor ceiling budget", then n_layers record
//           sizes, then n_layers*curve_len misses; prints the quotas of
//           plan_layer_quotas (src/h4/h4-cache-plan.cpp:146-223), or "E" when
//           it throws;
//   load:   "L <path>"; prints "P first last experts" and one line per curve of
//           CachePlan::load (src/h4/h4-cache-plan.cpp:31-86), or "E" when it
//           throws.

#include "h4-cache-plan.hpp"

#include <cstdio>
#include <iostream>
#include <string>
#include <vector>

using namespace galactus::h4;

int main() {
    std::string mode;
    while (std::cin >> mode) {
        if (mode == "Q") {
            std::size_t n = 0, len = 0;
            std::uint32_t floor = 0, ceiling = 0;
            std::uint64_t budget = 0;
            std::cin >> n >> len >> floor >> ceiling >> budget;
            std::vector<std::uint64_t> rec(n);
            for (auto & r : rec) std::cin >> r;
            std::vector<std::vector<std::uint32_t>> curves(n, std::vector<std::uint32_t>(len));
            for (auto & row : curves)
                for (auto & v : row) std::cin >> v;
            try {
                const auto q = plan_layer_quotas(curves, rec, budget, floor, ceiling);
                std::printf("R");
                for (auto v : q) std::printf(" %u", v);
                std::printf("\n");
            } catch (const std::exception &) {
                std::printf("E\n");
            }
        } else if (mode == "L") {
            std::string path;
            std::cin >> path;
            try {
                const CachePlan plan = CachePlan::load(path);
                std::printf("P %u %u %u\n", plan.first_layer, plan.last_layer, plan.experts);
                for (const auto & row : plan.curves) {
                    for (std::size_t i = 0; i < row.size(); ++i) std::printf(i ? " %u" : "%u", row[i]);
                    std::printf("\n");
                }
            } catch (const std::exception &) {
                std::printf("E\n");
            }
        }
        std::fflush(stdout);
    }
    return 0;
}
