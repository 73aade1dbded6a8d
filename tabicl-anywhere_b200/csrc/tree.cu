// The class tree of a member with more classes than the model tells apart (src/predict.rs:661-692): every node's
// scores become probabilities, the probabilities are multiplied down the tree, and the classes' products go back
// to scores.
#include <cfloat>

#include "kernels.cuh"

namespace tcu {

// One thread per test row. `nodes` are the tree's nodes in the order the reference's recursive walk visits them
// (a node before its children, children in map order): {k, leaf, offset of the node's scores in units of R, offset
// of its map}. A leaf's map entries are classes; an inner node's are the walk positions of its children, whose
// weights for this row are kept in wbuf[position][R]. Each node's scores are [R][k] at logits + offset * R.
__global__ void k_tree_combine(const float *__restrict__ logits, const int4 *__restrict__ nodes,
                               const int *__restrict__ map, int n_nodes, int R, int classes, float *__restrict__ wbuf,
                               float *__restrict__ out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    float *o = out + (size_t)r * classes;
    for (int c = 0; c < classes; c++) o[c] = 0.0f;
    for (int t = 0; t < n_nodes; t++) {
        const int4 nd = nodes[t];
        const int k = nd.x;
        const float w = t == 0 ? 1.0f : wbuf[(size_t)t * R + r];
        const float *sc = logits + (size_t)nd.z * R + (size_t)r * k;
        // predict.rs:669-674: the largest score (from f32::MIN, NaN ignored as f32::max does), exp((v - top) / 0.9)
        // summed in order, each divided by the sum
        float top = -FLT_MAX;
        for (int j = 0; j < k; j++) top = fmaxf(top, sc[j]);
        float sum = 0.0f;
        for (int j = 0; j < k; j++) sum += expf((sc[j] - top) / 0.9f);
        for (int j = 0; j < k; j++) {
            const float p = expf((sc[j] - top) / 0.9f) / sum;
            const int target = map[nd.w + j];
            // predict.rs:677-686: a leaf adds its share to its classes, an inner node hands weight * p down
            if (nd.y)
                o[target] += w * p;
            else
                wbuf[(size_t)target * R + r] = w * p;
        }
    }
    // predict.rs:690: back to scores
    for (int c = 0; c < classes; c++) o[c] = 0.9f * logf(o[c] + 1e-6f);
}

cudaError_t launch_tree_combine(const float *logits, const int4 *nodes, const int *map, int n_nodes, int R, int classes,
                                float *wbuf, float *out, cudaStream_t s, uint64_t *launches) {
    if (R <= 0) return cudaSuccess;
    k_tree_combine<<<(R + 127) / 128, 128, 0, s>>>(logits, nodes, map, n_nodes, R, classes, wbuf, out);
    if (launches) ++*launches;
    return cudaGetLastError();
}

}  // namespace tcu
