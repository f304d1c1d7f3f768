// placement.cu — where the routed experts of a mixture-of-experts model go on the GPUs of one node (b200_ep_place).
//
// speech.cpp places a Drama 3 model's routed experts between one GPU and the CPU: the GPU holds the experts of as many
// layers, from the first, as its free memory holds beside the rest of the model and its working memory, and the CPU
// computes the others (src/families/drama3/placement.cpp:58-74, src/engines/drama3-engine.cpp:51-88). On a B200 node
// the experts spread over the GPUs instead (expert parallelism): rank r of R holds experts [r E/R, (r+1) E/R) of every
// layer, and every rank holds the rest of the model (the router, attention and the other layers run replicated). The
// plan takes the fewest ranks (a power of two dividing E, at most the devices given) whose share fits each of the
// first R devices' free memory beside the rest, so the fewest ranks exchange partial sums; R = 1 is the single-device
// case. Host code only: it reads no device.
#include "internal.h"

extern "C" b200_status b200_ep_place(int n_devices, const size_t * free_bytes, int n_layers, const uint64_t * expert_bytes, int n_expert,
                                     uint64_t rest_bytes, b200_ep_plan * out) {
    if (!free_bytes || !out || n_devices < 1 || n_layers < 0 || (n_layers > 0 && !expert_bytes) || n_expert < 1) return B200_ERR_INVALID;
    uint64_t experts = 0;
    for (int l = 0; l < n_layers; l++) experts += expert_bytes[l];
    for (int ranks = 1; ranks <= n_devices && ranks <= kEpMaxRanks; ranks *= 2) {
        if (n_expert % ranks) break;
        // every layer's share, rounded up per layer (a layer's experts split evenly: each rank holds E / ranks of them)
        uint64_t share = 0;
        for (int l = 0; l < n_layers; l++) share += (expert_bytes[l] + (uint64_t) ranks - 1) / (uint64_t) ranks;
        bool fits = true;
        for (int d = 0; d < ranks && fits; d++) fits = rest_bytes + share <= (uint64_t) free_bytes[d];
        if (fits) {
            out->ranks = ranks;
            out->experts_per_rank = n_expert / ranks;
            out->bytes_per_rank = rest_bytes + share;
            out->expert_bytes = experts;
            return B200_OK;
        }
    }
    out->ranks = 0;
    out->experts_per_rank = 0;
    out->bytes_per_rank = 0;
    out->expert_bytes = experts;
    return B200_ERR_ALLOC;
}
