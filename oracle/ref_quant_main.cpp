// ref_quant_main.cpp -- runs the reference's own host quantizer on the CPU.
//
// TEST INFRASTRUCTURE ONLY (oracle side).  Compiled by oracle/build_oracle.py
// from the UNMODIFIED reference header src/quant_format.cuh where it lies;
// the binary goes to oracle/_ref/ref_quant and is never committed.
//
// quantize_weights_host (src/quant_format.cuh:58-116) ends by copying its host
// buffers to the device with cudaMalloc/cudaMemcpy.  Here those two calls (and
// cudaFree in free_quantized_weights, :118-123) are renamed at include time to
// host functions, so the reference's packing loop runs exactly as written and
// its results land in host memory.  No CUDA runtime is linked.
//
// usage: ref_quant <weights.f16> <d_out> <d_in> <out_prefix>
//   reads d_out*d_in binary16 values (row-major), writes
//   <out_prefix>.packed (u8 [d_out][d_in/2]), <out_prefix>.scales and
//   <out_prefix>.zeros (binary16 [d_out][d_in/128]).
#include <cuda_runtime.h>   // __device__/__forceinline__ and cudaError_t, as bindings.cpp does
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

template <class T>
static cudaError_t dq_host_malloc(T** p, size_t n) {
    *p = static_cast<T*>(std::malloc(n ? n : 1));
    return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
static cudaError_t dq_host_memcpy(void* d, const void* s, size_t n, cudaMemcpyKind) {
    std::memcpy(d, s, n);
    return cudaSuccess;
}
static cudaError_t dq_host_free(void* p) {
    std::free(p);
    return cudaSuccess;
}

#define cudaMalloc dq_host_malloc
#define cudaMemcpy dq_host_memcpy
#define cudaFree dq_host_free
#include "quant_format.cuh"
#undef cudaMalloc
#undef cudaMemcpy
#undef cudaFree

static bool write_file(const char* path, const void* p, size_t n) {
    FILE* f = std::fopen(path, "wb");
    if (!f) return false;
    bool ok = std::fwrite(p, 1, n, f) == n;
    return std::fclose(f) == 0 && ok;
}

int main(int argc, char** argv) {
    if (argc != 5) {
        std::fprintf(stderr, "usage: %s <weights.f16> <d_out> <d_in> <out_prefix>\n", argv[0]);
        return 2;
    }
    const int d_out = std::atoi(argv[2]);
    const int d_in = std::atoi(argv[3]);
    if (d_out <= 0 || d_in <= 0 || d_in % GROUP_SIZE) {
        std::fprintf(stderr, "bad shape %d x %d\n", d_out, d_in);
        return 2;
    }
    const size_t n = static_cast<size_t>(d_out) * d_in;
    std::vector<__half> w(n);
    FILE* f = std::fopen(argv[1], "rb");
    if (!f || std::fread(w.data(), sizeof(__half), n, f) != n) {
        std::fprintf(stderr, "cannot read %zu halfs from %s\n", n, argv[1]);
        return 2;
    }
    std::fclose(f);

    QuantizedWeights q = quantize_weights_host(w.data(), d_out, d_in);

    const size_t G = static_cast<size_t>(d_in) / GROUP_SIZE;
    std::string pre(argv[4]);
    bool ok = write_file((pre + ".packed").c_str(), q.packed, static_cast<size_t>(d_out) * (d_in / 2)) &&
              write_file((pre + ".scales").c_str(), q.scales, d_out * G * sizeof(__half)) &&
              write_file((pre + ".zeros").c_str(), q.zeros, d_out * G * sizeof(__half));
    free_quantized_weights(q);
    return ok ? 0 : 1;
}
