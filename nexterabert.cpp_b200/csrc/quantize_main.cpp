// nexterabert-quantize: the command line of the reference's tools/quantize.cpp on top of
// nextera_quantize (the block encoding runs on the GPU).
//
//   nexterabert-quantize in-f32.gguf out-Q4_K_M.gguf Q4_K_M [n_threads] [--tensor-type SUBSTRING=TYPE ...]
//
// n_threads is accepted for the same command lines and has no effect.
#include "nexterabert.h"

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

static void usage(const char * argv0) {
    fprintf(stderr, "usage: %s input.gguf output.gguf TYPE [n_threads] [--tensor-type SUBSTRING=TYPE ...]\n\n", argv0);
    fprintf(stderr, "file types: F32 F16 Q8_0 Q6_K Q5_K_M Q5_K_S Q5_0 Q4_K_M Q4_K_S Q4_0 Q3_K_M\n"
                    "--tensor-type overrides the type of every tensor whose name contains SUBSTRING\n"
                    "(tensor types: F32 F16 Q8_0 Q6_K Q5_K Q5_0 Q5_1 Q4_K Q4_0 Q4_1 Q3_K Q2_K).\n");
}

int main(int argc, char ** argv) {
    std::vector<std::string> pos, ovr;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (a == "--tensor-type" && i + 1 < argc) {
            ovr.push_back(argv[++i]);
        } else if (a == "-h" || a == "--help") {
            usage(argv[0]);
            return 0;
        } else {
            pos.push_back(a);
        }
    }
    if (pos.size() < 3) {
        usage(argv[0]);
        return 1;
    }
    std::vector<const char *> ov;
    for (const std::string & o : ovr) ov.push_back(o.c_str());
    const int32_t rc = nextera_quantize(pos[0].c_str(), pos[1].c_str(), pos[2].c_str(), (int32_t) ov.size(),
                                        ov.empty() ? nullptr : ov.data());
    return rc == 0 ? 0 : 1;
}
