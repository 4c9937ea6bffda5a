// Test program for include/tsrc_rt.hpp (driven by tests/test_rt_gpu.py): uploads a weight of the given
// host type from a file, runs linear() on activations from a file and writes y and the weight's device
// blocks (read_blocks) to files.
//   rt_check <dtype> <N> <K> <T> <x_stride> <max_part_k> <w.bin> <x.bin> <y.bin> <blocks.bin>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "tsrc_rt.hpp"

static std::vector<unsigned char> slurp(const char* p) {
    std::vector<unsigned char> v;
    if (FILE* f = std::fopen(p, "rb")) {
        unsigned char buf[65536];
        size_t n;
        while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) v.insert(v.end(), buf, buf + n);
        std::fclose(f);
    }
    return v;
}

static void spit(const char* p, const void* d, size_t n) {
    if (FILE* f = std::fopen(p, "wb")) {
        std::fwrite(d, 1, n, f);
        std::fclose(f);
    }
}

int main(int argc, char** argv) {
    if (argc != 11) return 2;
    const auto t = static_cast<tsrc::rt::dtype>(std::atoi(argv[1]));
    const uint32_t N = std::atoi(argv[2]), K = std::atoi(argv[3]), T = std::atoi(argv[4]);
    const size_t xs = std::atoi(argv[5]);
    tsrc::rt::weight_options o;
    o.max_part_k = std::atoi(argv[6]);
    const std::vector<unsigned char> w = slurp(argv[7]), x = slurp(argv[8]);
    try {
        tsrc::rt::device dev;
        const tsrc::rt::weight_handle h = dev.upload(t, w.data(), N, K, 0, o);
        const tsrc::rt::weight_info inf = dev.info(h);
        std::vector<float> y((size_t)T * N, -1.0f);
        dev.linear(h, reinterpret_cast<const float*>(x.data()), T, y.data(), xs, 0);
        const size_t rb = tsrc::rt::dtype_row_bytes(inf.fmt == TSRC_FMT_Q4_K ? tsrc::rt::dtype::q4_k : tsrc::rt::dtype::q8_0, K);
        std::vector<unsigned char> blocks(rb * N);
        dev.read_blocks(h, 0, N, blocks.data());
        spit(argv[9], y.data(), y.size() * sizeof(float));
        spit(argv[10], blocks.data(), blocks.size());
        std::printf("k_parts %u k_part %u fmt %u linears %llu\n", inf.k_parts, inf.k_part, inf.fmt,
                    (unsigned long long)dev.get_counters().linears);
        dev.free_weight(h);
        try {
            dev.free_weight(h);
            return 3;                                    // a freed handle must be refused
        } catch (const std::invalid_argument&) {
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    return 0;
}
