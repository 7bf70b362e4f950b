// moe.cuh — launch description of the device MoE layer (moe.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace strata {

// Per-expert assignment lists, written by the assignment kernel.
struct MoeIndex {
    int* cnt;       // [E] assignments routed to expert e (0 for experts not held here)
    int* off;       // [E] first sorted position of expert e
    int* active;    // [E] experts with cnt > 0, ascending; n_active of them
    int* n_active;  // [1]
    int* n_assign;  // [1] total assignments held here
    int* tok;       // [T k] token of each sorted assignment
    int* pos;       // [T k] sorted position of (token, slot), -1 when not held here
    // [slots] per grid slot: {expert, first sorted position, count, token of
    // the first assignment}, expert -1 past the active experts -- one load
    // gives a pass everything it needs to start streaming
    int4* slot_info;
    int slots;
};

struct MoePlan {
    int T, E, k, n_embd, n_ff, n_ff_s;
    int e_begin, e_end;  // experts held by this context (expert parallel): [e_begin, e_end)
    bool shared;         // run the shared expert here
    bool need_router;    // route from x through the router GEMV (no logits given)
    int slots;           // grid slots for active experts: min(T k, e_end - e_begin)
    int rc_gu, rc_d;     // row chunks of the gate/up and down passes
    int sm_count;
};

// Byte offsets of the workspace arrays.
struct MoeWork {
    int64_t ids, wts, pos, tok, cnt, off, active, counters, logits, xb, pgu, h, pd, gs, us, hs, gi, sg, ds, xfrag,
        xfrag_s, slot_info;
    int64_t bytes;
};

struct MoeTensor {
    uint32_t quant = 0;
    const uint8_t* W = nullptr;   // device bytes (experts: the first held expert)
    int64_t row_bytes = 0;
    int64_t expert_bytes = 0;     // rows * row_bytes for expert tensors
    const void* tmap = nullptr;   // tensor map of a dense Q4_K / Q5_K matrix (tensor-core GEMV), or null
};

struct MoeLaunch {
    MoePlan plan;
    MoeWork layout;
    void* work;                       // layout.bytes, 256-byte aligned
    const float* x;                   // [T][n_embd]
    const float* logits;              // [T][E] or null (then the router GEMV runs)
    float* out;                       // [T][n_embd]
    int* ids_out;                     // optional [T][k] device copies of the routing
    float* wts_out;
    int* err;                         // set by a kernel whose bounded wait expired
    MoeTensor router, gate, up, down, gate_s, up_s, down_s, gate_inp_s;
    // optional: the shared expert runs on `aux` (fork recorded on the caller's
    // stream, join waited on before the combine); null runs it in line
    cudaStream_t aux = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};

bool moe_expert_quant_supported(uint32_t q);
int moe_row_chunks(int slots, int mats, int IN, int sm_count, int T);
MoeWork moe_work_layout(const MoePlan& p);
int launch_moe_layer(const MoeLaunch& L, cudaStream_t s);

}  // namespace strata
