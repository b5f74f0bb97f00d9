// ddg_export_weights: writes the fixed-point weights.bin blob and its JSON
// manifest for the evaluators, in C++ so that a deployment needs no Python
// (restates reference/export_weights.py:27-75, dump_mpc_weights).
//
//   ddg_export_weights <scale> <weights.f32> <out.bin>
//
// <weights.f32>: the nine MPC layers of the affinity branch in forward order
// (gcn.0-2, drug_fc.0-1, fusion.0-3), each as its PyTorch weight (out, in)
// row-major float32 followed by its bias float32, little-endian, no header.
// <out.bin>: per layer W transposed to (in, out) row-major, then b, each
// value rint(x * 2^scale) (round half to even) as little-endian int64;
// <out.bin>.json: {scale, bitwidth 64, total_elements, layers: [{name,
// W_shape, b_shape, W_offset, b_offset}]} with the reference's key order and
// two-space indentation, so that the reference's loader
// (export_weights.py load_mpc_weights) and the evaluators read it unchanged.
// The evaluators shift b to scale 2 * scale when they load it
// (deepdtagen_inference.cu:169-178).  Exit status 0, 1 on usage, 2 on I/O errors.
#include <cfenv>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

namespace {

struct Layer {
    const char *name;
    int in, out;
};
// forward order, (in, out) of deepdtagen_inference.cu:113-123
const Layer kLayers[] = {{"gcn.0", 94, 188},       {"gcn.1", 188, 282},     {"gcn.2", 282, 376},
                         {"drug_fc.0", 376, 1024}, {"drug_fc.1", 1024, 128}, {"fusion.0", 256, 1024},
                         {"fusion.1", 1024, 512},  {"fusion.2", 512, 256},  {"fusion.3", 256, 1}};

int64_t to_fixed(float x, int scale)
{
    // x * 2^scale is exact in double; nearbyint rounds half to even like np.rint
    return int64_t(std::nearbyint(std::ldexp(double(x), scale)));
}

}  // namespace

int main(int argc, char **argv)
{
    if (argc != 4) {
        std::fprintf(stderr, "usage: ddg_export_weights <scale> <weights.f32> <out.bin>\n");
        return 1;
    }
    const int scale = std::atoi(argv[1]);
    if (scale < 0 || scale > 40) {
        std::fprintf(stderr, "ddg_export_weights: scale %d out of range\n", scale);
        return 1;
    }
    std::fesetround(FE_TONEAREST);
    size_t nfloat = 0;
    for (const Layer &l : kLayers) nfloat += size_t(l.in) * l.out + l.out;
    std::vector<float> w(nfloat);
    FILE *f = std::fopen(argv[2], "rb");
    if (!f) {
        std::fprintf(stderr, "ddg_export_weights: cannot open %s\n", argv[2]);
        return 2;
    }
    const size_t got = std::fread(w.data(), sizeof(float), nfloat, f);
    const bool extra = std::fgetc(f) != EOF;
    std::fclose(f);
    if (got != nfloat || extra) {
        std::fprintf(stderr, "ddg_export_weights: %s holds %s than the %zu float32 values of the nine layers\n",
                     argv[2], got != nfloat ? "fewer" : "more", nfloat);
        return 2;
    }
    std::vector<int64_t> blob;
    blob.reserve(nfloat);
    std::string layers_json;
    size_t src = 0;
    for (size_t li = 0; li < sizeof(kLayers) / sizeof(kLayers[0]); li++) {
        const Layer &l = kLayers[li];
        const size_t w_off = blob.size();
        // PyTorch (out, in) -> (in, out)
        for (int i = 0; i < l.in; i++)
            for (int o = 0; o < l.out; o++) blob.push_back(to_fixed(w[src + size_t(o) * l.in + i], scale));
        src += size_t(l.in) * l.out;
        const size_t b_off = blob.size();
        for (int o = 0; o < l.out; o++) blob.push_back(to_fixed(w[src + o], scale));
        src += l.out;
        char buf[512];
        std::snprintf(buf, sizeof(buf),
                      "%s    {\n      \"name\": \"%s\",\n      \"W_shape\": [\n        %d,\n        %d\n      ],\n"
                      "      \"b_shape\": [\n        %d\n      ],\n      \"W_offset\": %zu,\n      \"b_offset\": %zu\n"
                      "    }",
                      li ? ",\n" : "", l.name, l.in, l.out, l.out, w_off, b_off);
        layers_json += buf;
    }
    FILE *o = std::fopen(argv[3], "wb");
    if (!o || std::fwrite(blob.data(), sizeof(int64_t), blob.size(), o) != blob.size()) {
        std::fprintf(stderr, "ddg_export_weights: cannot write %s\n", argv[3]);
        if (o) std::fclose(o);
        return 2;
    }
    std::fclose(o);
    const std::string jpath = std::string(argv[3]) + ".json";
    FILE *j = std::fopen(jpath.c_str(), "w");
    if (!j) {
        std::fprintf(stderr, "ddg_export_weights: cannot write %s\n", jpath.c_str());
        return 2;
    }
    std::fprintf(j, "{\n  \"scale\": %d,\n  \"bitwidth\": 64,\n  \"total_elements\": %zu,\n  \"layers\": [\n%s\n  ]\n}",
                 scale, blob.size(), layers_json.c_str());
    std::fclose(j);
    return 0;
}
