// Prints what trochilus_b200/csrc/gguf_file.h reads from a GGUF file: the status, then one line per tensor
// (name, ggml type, dimensions, absolute offset, bytes) and the olmoe.* integers. Built and run by tests/test_gguf.py,
// in a child process, so that a malformed file can only end this program, never the test run.
#include <cstdio>
#include <string>

#include "../trochilus_b200/csrc/gguf_file.h"

int main(int argc, char **argv) {
    if (argc < 2) return 2;
    TrxGguf g;
    std::string err;
    if (!g.open(argv[1], err)) {
        printf("error %s\n", err.c_str());
        return 1;
    }
    printf("ok %u\n", g.version());
    for (int i = 2; i < argc; i++) {
        const TrxGgufTensor *t = g.tensor(argv[i]);
        if (t == nullptr) {
            printf("absent %s\n", argv[i]);
            continue;
        }
        printf("tensor %s %u %u", t->name.c_str(), t->type, t->n_dims);
        for (uint32_t d = 0; d < t->n_dims; d++) printf(" %llu", (unsigned long long)t->ne[d]);
        printf(" @ %llu %llu\n", (unsigned long long)t->offset, (unsigned long long)t->n_bytes);
    }
    uint32_t v = 0;
    if (g.get_u32("olmoe.expert_count", v)) printf("expert_count %u\n", v);
    return 0;
}
