// fused.h — fused multi-gate passes over shared-memory tiles (host + device layouts).
//
// A pass loads a tile of 2^k amplitudes whose tile-local index bit j is global qubit S[j]
// (S sorted, S[0..L) = 0..L-1 so a tile is 2^(k-L) contiguous runs of 2^L amplitudes), applies a
// sequence of gates whose non-diagonal targets lie in S, and writes the tile back: one HBM read
// and write of the state for the whole sequence. Diagonal gates and controls may sit on any
// qubit (their bits are known per tile). Inside the tile the gates are grouped in sub-blocks: each
// thread holds 2^RB amplitudes in registers spanning RB "register bits" R of the tile, applies
// every gate of the sub-block whose targets lie in R, and the tile round-trips through shared
// memory only between sub-blocks.
//
// Shared-memory layout: tile element j lives at phys(j) = j ^ fold(j), where fold XORs the
// 3-bit groups j[3:6], j[6:9], j[9:12] into the low 3 bits. A quarter-warp (8 lanes) whose
// lane bits map to tile bits with distinct residues mod 3 touches 8 distinct 16-byte bank slots.
#pragma once

#ifndef __CUDACC_RTC__
#include <stdint.h>
#endif

namespace arcqml {

constexpr int kTileMax = 12;       // tile qubits
constexpr int kLowFixed = 4;       // S always holds qubits 0..kLowFixed-1 (256-byte runs)
constexpr int kMaxPassOps = 256;   // fused ops per pass (staged in shared memory)
constexpr int kMaxPassMats = 1536; // matrix-table entries (double2) per pass
constexpr int kMaxPassAcc = 56;    // gradient accumulators per pass (one smem column per thread)

enum FusedKind : uint8_t {
    FK_M2 = 0,  // dense 2x2 on register bit rb0; m = [m00 m01 m10 m11]
    FK_RX = 1,  // m[0] = (c, s): [[c, -is], [-is, c]]
    FK_RY = 2,  // m[0] = (c, s): [[c, -s], [s, c]]
    FK_D1 = 3,  // diagonal (d0, d1) on one qubit anywhere
    FK_D2 = 4,  // diagonal (d0..d3) on two qubits anywhere, index bit(q0) + 2 bit(q1)
    FK_M4 = 5,  // dense 4x4 on register bits (rb0, rb1)
};

enum GradKind : uint8_t {
    GK_NONE = 0,
    GK_PX = 1,       // rotation about X on rb0: slot gradient = Im<lam|X|psi> (psi before U^dag)
    GK_PY = 2,       // about Y
    GK_PZ = 3,       // about Z on a diag qubit (dq 0)
    GK_GENERIC = 4,  // per slot: Re<lam| dU_s |psi'> with psi' = U^dag psi (dU after U's matrix)
};

// Specialised code paths the planner selects per op (the generic path handles every case;
// the others are exact rewrites for common shapes without per-element control logic).
enum FastCode : uint8_t {
    FC_GENERIC = 0,  // kind + controls, evaluated per element
    FC_RX = 1,       // uncontrolled RX-form on register bit rb0
    FC_RY = 2,       // uncontrolled RY-form on register bit rb0
    FC_M2 = 3,       // uncontrolled 2x2 on register bit rb0
    FC_D1_REG = 4,   // uncontrolled diagonal on register bit rb0
    FC_D1_UNI = 5,   // uncontrolled diagonal on a qubit constant per thread (dq 0)
    FC_SIGN_RR = 6,  // -1 where register bits rb0 and rb1 are both set (CZ)
    FC_SIGN_RC = 7,  // -1 where register bit rb0 and the per-thread bit dq 0 are set
    FC_SIGN_CC = 8,  // -1 where the per-thread bits dq 0 and dq 1 are set
    FC_M4 = 9,       // uncontrolled 4x4 on register bits (rb0, rb1)
    FC_X = 10,       // uncontrolled X on register bit rb0 (register renaming)
    FC_CX_RR = 11,   // X on register bit rb0 where register bit rb1 (the control) is 1
    FC_CX_CR = 12,   // X on register bit rb0 where the per-thread bit dq 0 (the control) is 1
    // Run-time compiled kernels only (on unless ARCQML_FAST_DIAG=0): each qubit of the op (diagonal
    // slots, controls) is a register bit or a per-thread value, resolved when the code is
    // generated; the table-driven kernel runs these codes through its generic path.
    FC_DIAG = 13,    // diagonal (FK_D1 / FK_D2) with any controls
    FC_CM2 = 14,     // one-target gate (FK_RX / FK_RY / FK_M2) on rb0 with controls
};

enum GradFast : uint8_t {
    GF_GENERIC = 0,  // gkind path with per-element control logic
    GF_X = 1,        // uncontrolled Im<lam|X_rb0|psi>
    GF_Y = 2,        // uncontrolled Im<lam|Y_rb0|psi>
    GF_Z_REG = 3,    // uncontrolled Im<lam|Z_rb0|psi>
    GF_Z_UNI = 4,    // uncontrolled Im<lam|Z|psi> on the per-thread bit dq 0
};

struct FOp {
    uint8_t kind;
    uint8_t rb0, rb1;        // register bits of the targets (FK_M2/RX/RY/M4)
    uint8_t gkind;           // adjoint passes only
    uint8_t dq_in_tile[2];   // FK_D1/FK_D2: qubit lies in the tile
    uint8_t dq_pos[2];       // tile-local bit if in the tile, else global position
    uint16_t lcmask;         // controls inside the tile (tile-local bits)
    uint16_t nslots;         // GK_GENERIC: number of slots
    uint32_t moff;           // offset of the op's matrices in the pass matrix table
    uint32_t acc[3];         // pass-local accumulator index per slot
    uint8_t code;            // FastCode
    uint8_t gcode;           // GradFast
    uint8_t sform;           // compiled passes: apply the unit-diagonal form of mats[soff]
    uint8_t sgrad;           // compiled passes: gradient factor in mats[soff].y
    uint64_t gcmask;         // controls outside the tile (global positions)
    uint32_t soff;           // scaled-pass entry: (tau, 0.5 |sigma|^2 before the op)
    uint32_t pad[5];
};
static_assert(sizeof(FOp) == 64, "FOp layout");

struct SubBlock {
    uint8_t R[4];            // register bits (tile-local), ascending; RB of them are used
    uint8_t perm[12];        // thread bit i -> tile-local bit perm[i] (the bits not in R)
    uint16_t op_begin, op_end;
    uint32_t flags;          // SB_ALL_FAST: every op of the sub-block has a fast path
};
constexpr uint32_t SB_ALL_FAST = 1;  // the table-driven kernel has a fast path for every op
constexpr uint32_t SB_JIT_FAST = 2;  // the run-time compiled kernels have one for every op
constexpr uint32_t SB_WARP_NEXT = 4; // the next sub-block keeps every element in the same warp
static_assert(sizeof(SubBlock) == 24, "SubBlock layout");

// Row stride of a pass's accumulator table (doubles, shared memory) for `cols` columns, one per
// `lanes` threads. Kernels that reduce a gradient over four lanes first (accumulate_quad2)
// update two rows, usually consecutive ones, in one access: a stride of cols + 8 puts row a + 1
// in the other half of the banks, where a stride of 64 (512 bytes) would give a two-way conflict.
#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
__host__ __device__
#endif
constexpr uint32_t acc_row_stride(uint32_t cols, uint32_t lanes) {
    return lanes == 4u ? cols + 8u : cols;
}

struct PassHeader {
    uint32_t k;              // tile bits
    uint32_t nsub;
    uint32_t nops;
    uint32_t nmat;           // double2 entries
    uint32_t nacc;           // accumulators used (adjoint)
    uint32_t acc_base;       // first global accumulator row of this pass
    uint32_t rb;             // register bits per thread (3 or 4)
    uint32_t pad0;
    uint8_t S[16];           // tile bit -> global qubit
};
static_assert(sizeof(PassHeader) == 48, "PassHeader layout");

}  // namespace arcqml
