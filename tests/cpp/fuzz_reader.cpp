// fuzz_reader.cpp — the checkpoint reader's parsing paths under AddressSanitizer
// and UndefinedBehaviorSanitizer (built with g++ by tests/cpp/Makefile, target
// fuzz_reader; driven by tests/test_loader_fuzz.py).  Checkpoint files are
// untrusted input: whatever their bytes, SafetensorsReader::load must either
// refuse them or describe tensors that lie inside the file, and the JSON
// reader must accept or reject every line without reading out of bounds.
//
//   fuzz_reader files <path>...   load each file; on success read every byte
//                                 of every tensor through get_raw_ptr
//   fuzz_reader json <path>       parse each line of the file
// No CUDA call is made.  Prints one summary line; exit status 0 unless a
// sanitizer stops the process.
#include <cstdint>
#include <cstdio>
#include <fstream>
#include <iostream>
#include <string>

#include "json_lite.h"
#include "model_loaders/safetensors_loader.h"

using namespace hxinfer;

int main(int argc, char** argv)
{
    if (argc < 3) {
        std::cerr << "usage: fuzz_reader files <path>... | json <path>\n";
        return 2;
    }
    const std::string mode = argv[1];
    if (mode == "json") {
        std::ifstream f(argv[2], std::ios::binary);
        std::string line;
        long ok = 0, bad = 0;
        while (std::getline(f, line)) {
            json_lite::Value v;
            std::string err;
            (json_lite::parse(line.data(), line.data() + line.size(), v, &err) ? ok : bad)++;
        }
        std::cout << "json ok " << ok << " rejected " << bad << "\n";
        return 0;
    }
    long loaded = 0, refused = 0, tensors = 0;
    uint64_t checksum = 0;
    for (int i = 2; i < argc; ++i) {
        SafetensorsReader r;
        if (!r.load(argv[i])) {
            ++refused;
            continue;
        }
        ++loaded;
        for (const auto& name : r.tensor_names()) {
            const SafetensorInfo* info = r.get_info(name);
            const unsigned char* p = static_cast<const unsigned char*>(r.get_raw_ptr(name));
            for (size_t b = info->offset_begin; b < info->offset_end; ++b) checksum += p[b - info->offset_begin];
            ++tensors;
        }
    }
    std::cout << "files loaded " << loaded << " refused " << refused << " tensors " << tensors
              << " checksum " << checksum << "\n";
    return 0;
}
