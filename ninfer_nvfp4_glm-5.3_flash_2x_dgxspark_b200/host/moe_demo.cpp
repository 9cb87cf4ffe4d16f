// moe_demo.cpp -- a C++ host running one feed-forward layer through
// nf_host::MoeLayer (or nf_host::DenseMlp): reads a tensor store (checkpoint
// names, the reference's tensor kinds), binds the layer by name, runs
// TextModel::moe's (or dense_mlp's) contract over the token rows `x` and
// writes y.  It stands where the reference's own host would sit.
//
// usage: moe_demo <store> <prefix> <out_y.f32> hidden experts top_k inter shared_inter
//                 routed_scaling [device]
// store: a safetensors checkpoint directory (model.safetensors.index.json and
// its shards, or model.safetensors: nf_host::SafetensorsStore), or a tensor
// file: "NFT1", then records {u32 name_len, name, u8 kind, u32 rank, i64
// dims[rank], u64 bytes, data}.  The store holds `x`, F32 [tokens, hidden].
// experts == 0 runs the dense MLP of the first layers (hidden, inter).
#include "nf_moe_layer.hpp"
#include "nf_safetensors.hpp"

#include <sys/stat.h>
#include <unistd.h>

#include <chrono>
#include <thread>

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <map>
#include <string>
#include <vector>

namespace {

struct Record {
    nf_host::TensorView view;
    std::vector<unsigned char> bytes;
};

std::map<std::string, Record> read_tensors(const char* path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error(std::string("cannot open ") + path);
    char magic[4];
    in.read(magic, 4);
    if (!in || std::memcmp(magic, "NFT1", 4) != 0) throw std::runtime_error("not a tensor file");
    std::map<std::string, Record> out;
    for (;;) {
        uint32_t n = 0;
        if (!in.read(reinterpret_cast<char*>(&n), 4)) break;
        std::string name(n, '\0');
        in.read(&name[0], n);
        unsigned char kind = 0;
        uint32_t rank = 0;
        in.read(reinterpret_cast<char*>(&kind), 1);
        in.read(reinterpret_cast<char*>(&rank), 4);
        Record r;
        r.view.kind = static_cast<char>(kind);
        r.view.shape.resize(rank);
        in.read(reinterpret_cast<char*>(r.view.shape.data()), static_cast<std::streamsize>(8 * rank));
        uint64_t bytes = 0;
        in.read(reinterpret_cast<char*>(&bytes), 8);
        r.bytes.resize(bytes);
        in.read(reinterpret_cast<char*>(r.bytes.data()), static_cast<std::streamsize>(bytes));
        if (!in) throw std::runtime_error("truncated tensor " + name);
        out.emplace(name, std::move(r));
    }
    for (auto& kv : out) kv.second.view.data = kv.second.bytes.data();
    return out;
}

}  // namespace

// The group id of an expert-parallel run: rank 0 makes it and publishes it as
// a file (written then renamed, so a reader sees it whole); the other ranks
// wait for the file (two minutes at most).
std::vector<uint8_t> ep_group_id(int rank, const std::string& path) {
    std::vector<uint8_t> id(NF_EP_ID_BYTES);
    if (rank == 0) {
        if (nf_ep_unique_id(id.data(), NF_EP_ID_BYTES) != NF_OK) throw std::runtime_error("nf_ep_unique_id failed");
        const std::string tmp = path + ".tmp";
        {
            std::ofstream f(tmp, std::ios::binary);
            f.write(reinterpret_cast<const char*>(id.data()), NF_EP_ID_BYTES);
            if (!f) throw std::runtime_error("cannot write " + tmp);
        }
        if (std::rename(tmp.c_str(), path.c_str()) != 0) throw std::runtime_error("cannot publish " + path);
        return id;
    }
    for (int i = 0; i < 2400; ++i) {
        std::ifstream f(path, std::ios::binary);
        if (f && f.read(reinterpret_cast<char*>(id.data()), NF_EP_ID_BYTES)) return id;
        std::this_thread::sleep_for(std::chrono::milliseconds(50));
    }
    throw std::runtime_error("no group id at " + path);
}

int main(int argc, char** argv) {
    if (argc < 10) {
        std::fprintf(stderr,
                     "usage: %s tensors.nft prefix out_y.f32 hidden experts top_k inter shared_inter scaling [device "
                     "[--ep rank world group_id_file]]\n",
                     argv[0]);
        return 2;
    }
    try {
        struct stat st {};
        const bool is_dir = ::stat(argv[1], &st) == 0 && S_ISDIR(st.st_mode);
        std::unique_ptr<nf_host::SafetensorsStore> ckpt;
        std::map<std::string, Record> records;
        nf_host::StoreLookup lookup;
        if (is_dir) {
            ckpt = std::make_unique<nf_host::SafetensorsStore>(argv[1]);
            lookup = ckpt->lookup();
            std::printf("moe_demo: %zu tensors in %zu shards, %llu bytes mapped\n", ckpt->tensor_count(),
                        ckpt->shard_count(), static_cast<unsigned long long>(ckpt->data_bytes()));
        } else {
            records = read_tensors(argv[1]);
            lookup = [&records](const std::string& name) -> const nf_host::TensorView* {
                const auto it = records.find(name);
                return it == records.end() ? nullptr : &it->second.view;
            };
        }
        const std::string prefix = argv[2];
        const nf_host::TensorView* x = lookup("x");
        if (!x || x->kind != 'f' || x->shape.size() != 2) throw std::runtime_error("missing tensor x");
        nf_moe_desc d{};
        d.hidden = std::atoi(argv[4]);
        d.experts = std::atoi(argv[5]);
        d.top_k = std::atoi(argv[6]);
        d.inter = std::atoi(argv[7]);
        d.shared_inter = std::atoi(argv[8]);
        d.n_group = 1;
        d.topk_group = 1;
        d.normalize = 1;
        d.routed_scaling = static_cast<float>(std::atof(argv[9]));
        d.swiglu_limit = 10.f;
        d.expert_kind = NF_EXPERTS_NVFP4;
        d.max_tokens = static_cast<int>(x->dim(0));
        const int device = argc > 10 ? std::atoi(argv[10]) : 0;
        std::vector<float> y(static_cast<size_t>(x->dim(0) * x->dim(1)));
        if (argc > 11 && std::strcmp(argv[11], "--ep") == 0) {
            // expert parallel: this rank's handle, its share of the token rows
            // (rows [T r / world, T (r + 1) / world)), out_y gets those rows
            if (argc < 15) throw std::runtime_error("--ep needs rank world group_id_file");
            const int rank = std::atoi(argv[12]), world = std::atoi(argv[13]);
            const int64_t T = x->dim(0), H = x->dim(1);
            const int64_t r0 = T * rank / world, r1 = T * (rank + 1) / world;
            d.max_tokens = static_cast<int>((T + world - 1) / world);
            const std::vector<uint8_t> id = ep_group_id(rank, argv[14]);
            nf_host::MoeLayer layer(d, device, rank, world, id.data(), NF_EP_ID_BYTES);
            layer.bind_from_store(lookup, prefix);
            layer.moe(static_cast<const float*>(x->data) + r0 * H, y.data() + r0 * H, static_cast<int>(r1 - r0));
            std::ofstream out(argv[3], std::ios::binary);
            out.write(reinterpret_cast<const char*>(y.data() + r0 * H), static_cast<std::streamsize>((r1 - r0) * H * 4));
            std::printf("moe_demo: rank %d of %d (%s), rows %lld-%lld\n", rank, world, layer.ep_transport(),
                        static_cast<long long>(r0), static_cast<long long>(r1));
            return 0;
        }
        if (d.experts == 0) {
            nf_host::DenseMlp mlp(d.hidden, d.inter, d.swiglu_limit, d.max_tokens, device);
            mlp.bind_from_store(lookup, prefix);
            mlp.dense_mlp(static_cast<const float*>(x->data), y.data(), static_cast<int>(x->dim(0)));
        } else {
            nf_host::MoeLayer layer(d, device);
            layer.bind_from_store(lookup, prefix);
            layer.moe(static_cast<const float*>(x->data), y.data(), static_cast<int>(x->dim(0)));
        }
        std::ofstream out(argv[3], std::ios::binary);
        out.write(reinterpret_cast<const char*>(y.data()), static_cast<std::streamsize>(y.size() * 4));
        double sum = 0;
        for (float v : y) sum += v;
        std::printf("moe_demo: %lld tokens, checksum %.9g\n", static_cast<long long>(x->dim(0)), sum);
    } catch (const std::exception& e) {
        std::fprintf(stderr, "moe_demo: %s\n", e.what());
        return 1;
    }
    return 0;
}
