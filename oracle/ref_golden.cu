// ref_golden.cu -- TEST INFRASTRUCTURE ONLY. Builds the reference harness's own host-side input
// generator and reference reduction (collectives/harness/main.cu: fill_input :118-126, reference
// :129-149) straight from the reference sources: main.cu is included with its main() renamed, so no
// GPU code of the reference ever runs. One binary per compile-time (COLL_OP, CLUSTER_N, MSG_ELEMS,
// ELEM_T), exactly like the reference build matrix. Built by oracle/Makefile into oracle/_ref/.
//
//   <bin> golden A|B <file>           write the golden record (header, input, reference output)
//   <bin> bench <seconds> <threads>   time reference() (the reference's CPU path) on `threads` host
//                                     threads, each on its own problem, for ~<seconds>; prints JSON
#define main dsmem_reference_harness_main
#include REFERENCE_HARNESS
#undef main

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

static int write_golden(char pattern, const char* path) {
    std::vector<ELEM_T> in(kInElems);
    fill_input(in, pattern);
    const std::vector<double> ref = reference(in);
    FILE* f = std::fopen(path, "wb");
    if (f == nullptr) return 2;
    const long long hdr[6] = {(long long)COLL_OP, (long long)CLUSTER_N, (long long)MSG_ELEMS, (long long)kIsInt,
                              (long long)in.size(), (long long)ref.size()};
    std::fwrite(hdr, sizeof hdr, 1, f);
    std::fwrite(in.data(), sizeof(ELEM_T), in.size(), f);
    std::fwrite(ref.data(), sizeof(double), ref.size(), f);
    std::fclose(f);
    return 0;
}

static int bench(double seconds, int threads) {
    std::vector<std::vector<ELEM_T>> ins(threads, std::vector<ELEM_T>(kInElems));
    for (int t = 0; t < threads; ++t) fill_input(ins[t], 'B');
    std::atomic<long long> problems{0};
    std::atomic<bool> stop{false};
    double sink = 0.0;
    std::vector<double> sinks(threads, 0.0);
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t)
        pool.emplace_back([&, t] {
            long long n = 0;
            while (!stop.load(std::memory_order_relaxed)) {
                const std::vector<double> r = reference(ins[t]);
                sinks[t] += r[n % r.size()];
                ++n;
                if ((n & 15) == 0 &&
                    std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > seconds)
                    stop = true;
            }
            problems += n;
        });
    for (auto& th : pool) th.join();
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    for (double s : sinks) sink += s;
    std::printf("{\"problems\": %lld, \"seconds\": %.6f, \"threads\": %d, \"payload_bytes\": %zu, \"sink\": %.3f}\n",
                problems.load(), el, threads, (size_t)kPayloadBytes, sink);
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 4 && std::strcmp(argv[1], "golden") == 0) return write_golden(argv[2][0], argv[3]);
    if (argc >= 4 && std::strcmp(argv[1], "bench") == 0) return bench(std::atof(argv[2]), std::atoi(argv[3]));
    std::fprintf(stderr, "usage: %s golden A|B <file> | bench <seconds> <threads>\n", argv[0]);
    return 1;
}
