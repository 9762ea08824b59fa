// SPDX-License-Identifier: Apache-2.0
// Smallest use of the library: a 2x3 by 3x2 FP64 product through ozTTgemm::Context, checked
// against its exact value. The options pick the first available format (INT8 on B200).
#include <ozTTgemm/ozTTgemm.hpp>

#include <iostream>
#include <vector>

int main() {
    try {
        ozTTgemm::Options options;
        options.scheme = ozTTgemm::Scheme::II;
        for (auto f : {ozTTgemm::Format::BFP8, ozTTgemm::Format::BF16, ozTTgemm::Format::FP16, ozTTgemm::Format::TF32,
                       ozTTgemm::Format::FP8, ozTTgemm::Format::INT8})
            if (ozTTgemm::is_available(f)) {
                options.format = f;
                break;
            }
        ozTTgemm::Context context;
        const std::vector<double> a{1, 2, 3, 4, 5, 6};     // 2 x 3, row-major
        const std::vector<double> b{7, 8, 9, 10, 11, 12};  // 3 x 2
        const std::vector<double> c = context.multiply(a, b, 2, 2, 3, options);
        std::cout << c[0] << ' ' << c[1] << '\n' << c[2] << ' ' << c[3] << '\n';
        return c == std::vector<double>{58, 64, 139, 154} ? 0 : 1;
    } catch (const std::exception& e) {
        std::cerr << e.what() << '\n';
        return 1;
    }
}
