// sharded.h — jhq::ShardedIndex: one process, several shards (GPUs, or
// several shards on one GPU), behind the reference's JHQGpuIndex call shape
// (jhq_v14_streaming_add/jhq_gpu_index.cuh:14-83); the reference itself is
// single-GPU.
//
// Vectors are placed round-robin by global id: id g lives on shard g % S as
// local id g / S, so ids need no map and repeated add() calls keep the rule.
// All shards hold the same trained artefacts (shard 0 trains, the others
// import its artefacts and its pilot clusters), so probe choices agree everywhere.
//
// search(), per chunk of queries:
//   1. the queries go to every shard's device;
//   2. coarse step split by queries: non-empty shard r computes the probe
//      lists of its 1/R of the chunk (rotation + coarse scores + top-nprobe)
//      and the slices are copied to every other shard (peer copies);
//   3. every non-empty shard scans its vectors with those lists and keeps
//      its top-k, local ids turned into global ids on its own device;
//   4. the R lists are copied to the first shard's device and merged there
//      by (distance, id) (merge_shard_lists), then copied to the host.
// Each shard keeps its own exact top-ck before its residual refine, so the
// candidate set is a superset of a single index's (results are not
// bit-identical to one index holding all vectors; they are bit-identical to
// searching the shards one by one and merging).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <vector>

#include "index.h"
#include "jhq_common.h"

namespace jhq {

class ShardedIndex {
public:
    ShardedIndex(int d, const Params& p, const std::vector<int>& devices);
    ~ShardedIndex();
    ShardedIndex(const ShardedIndex&) = delete;
    ShardedIndex& operator=(const ShardedIndex&) = delete;

    void train(const float* h_x, int64_t n);
    void add(const float* h_x, int64_t n);
    void search(const float* h_q, int64_t nq, int k, float* h_dists, int32_t* h_ids);
    void set_nprobe(int nprobe);

    int64_t ntotal() const { return ntotal_; }
    int nshards() const { return (int)sh_.size(); }
    bool trained() const { return sh_[0]->trained(); }
    Index& shard(int s) { return *sh_[s]; }

private:
    struct ShardBufs {
        int dev = 0;
        cudaStream_t st = nullptr;
        cudaEvent_t ev_probe = nullptr, ev_done = nullptr;
        DevBuf<float> q, D;
        DevBuf<int32_t> I, probes;
    };
    void sync_artefacts();

    int d_;
    Params p_;
    std::vector<std::unique_ptr<Index>> sh_;
    std::vector<ShardBufs> b_;
    int64_t ntotal_ = 0;
    DevBuf<float> allD_, outD_;          // on shard 0's device
    DevBuf<int32_t> allI_, outI_;
    PinnedBuf<float> hq_, hD_;
    PinnedBuf<int32_t> hI_;
};

}  // namespace jhq
