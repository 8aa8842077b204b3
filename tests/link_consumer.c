/* link_consumer.c — a C program linked against the static archive the way the Rust crate
 * arcqml-runtime-sys links it (crates/arcqml-runtime-sys/build.rs:10-21: static library
 * arcqml_runtime_private, plus the CUDA runtime and C++ library the archive needs), calling the
 * v1 entry points exactly as crates/arcqml-runtime-sys/src/lib.rs:265-313 does.
 *
 *   link_consumer check
 *       ABI version, plan create / push / destroy and the last-error protocol (no GPU needed).
 *   link_consumer run <input> <output>
 *       reads a plan, upstream factor, requires-grad mask, initial state and adjoint state;
 *       runs arcqml_rt_v1_circuit_plan_apply on the initial state, then
 *       arcqml_rt_v1_adjoint_backward on (final state, adjoint state); writes the final state,
 *       the state and adjoint state after the sweep, and the gradients.
 *
 * Input (little-endian): u32 n, u32 nops; per op: u32 opcode, u32 arity, f64 params[3],
 * u64 qubits[arity], u32 nbindings, nbindings x (u64 slot, u64 parent); u64 nreq,
 * u8 req[nreq]; f64 upstream; c128 init[2^n]; c128 lambda[2^n].
 * Output: c128 final[2^n], c128 psi0[2^n], c128 lambda0[2^n], f64 grads[nreq].
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "arcqml_runtime.h"

static void last_error(const char *what) {
    size_t len = arcqml_rt_last_error(NULL, 0);
    uint8_t *buf = (uint8_t *)calloc(len + 1, 1);
    if (buf) arcqml_rt_last_error(buf, len + 1);
    fprintf(stderr, "%s failed: %s\n", what, buf ? (const char *)buf : "?");
    free(buf);
}

static int rd(FILE *f, void *p, size_t n) { return fread(p, 1, n, f) == n ? 0 : -1; }

static int check(void) {
    if (arcqml_rt_abi_version() != ARCQML_RT_ABI_VERSION) return 2;
    CircuitPlanHandle plan = {NULL};
    if (arcqml_rt_v1_circuit_plan_create_empty(4, &plan) != 0) return 3;
    const size_t q[2] = {0, 1};
    GateDescriptor g;
    memset(&g, 0, sizeof g);
    g.abi_version = ARCQML_RT_ABI_VERSION;
    g.opcode = ARCQML_OP_RY;
    g.arity = 1;
    OperationDescriptor op;
    memset(&op, 0, sizeof op);
    op.gate = g;
    op.qubits = q;
    op.qubits_len = 2; /* arity 1 with two qubits: rejected */
    if (arcqml_rt_v1_circuit_plan_push(&plan, &op) == 0) return 4;
    size_t len = arcqml_rt_last_error(NULL, 0);
    uint8_t *msg = (uint8_t *)calloc(len + 1, 1);
    if (!msg || len == 0) return 5;
    arcqml_rt_last_error(msg, len + 1);
    op.qubits_len = 1;
    if (arcqml_rt_v1_circuit_plan_push(&plan, &op) != 0) return 6;
    arcqml_rt_v1_circuit_plan_destroy(&plan);
    arcqml_rt_v1_circuit_plan_destroy(&plan); /* idempotent */
    printf("abi %u\nerror %s\n", arcqml_rt_abi_version(), (const char *)msg);
    free(msg);
    return 0;
}

static int run(const char *in_path, const char *out_path) {
    FILE *f = fopen(in_path, "rb");
    if (!f) return 10;
    uint32_t n = 0, nops = 0;
    if (rd(f, &n, 4) || rd(f, &nops, 4) || n == 0 || n > 30) return 11;
    CircuitPlanHandle plan = {NULL};
    if (arcqml_rt_v1_circuit_plan_create_empty(nops, &plan) != 0) {
        last_error("plan_create_empty");
        return 12;
    }
    for (uint32_t i = 0; i < nops; ++i) {
        uint32_t opcode = 0, arity = 0, nb = 0;
        double params[3];
        size_t qubits[8];
        ParameterBindingDescriptor b[3];
        if (rd(f, &opcode, 4) || rd(f, &arity, 4) || arity == 0 || arity > 8 ||
            rd(f, params, sizeof params))
            return 13;
        for (uint32_t j = 0; j < arity; ++j) {
            uint64_t q = 0;
            if (rd(f, &q, 8)) return 13;
            qubits[j] = (size_t)q;
        }
        if (rd(f, &nb, 4) || nb > 3) return 13;
        for (uint32_t j = 0; j < nb; ++j) {
            uint64_t s = 0, p = 0;
            if (rd(f, &s, 8) || rd(f, &p, 8)) return 13;
            b[j].parameter_slot = (size_t)s;
            b[j].parent_index = (size_t)p;
        }
        OperationDescriptor op;
        memset(&op, 0, sizeof op);
        op.gate.abi_version = ARCQML_RT_ABI_VERSION;
        op.gate.opcode = opcode;
        op.gate.arity = arity;
        memcpy(op.gate.parameters, params, sizeof params);
        op.qubits = qubits;
        op.qubits_len = arity;
        op.parameters = nb ? b : NULL;
        op.parameters_len = nb;
        if (arcqml_rt_v1_circuit_plan_push(&plan, &op) != 0) {
            last_error("plan_push");
            return 14;
        }
    }
    uint64_t nreq = 0;
    double upstream = 0.0;
    if (rd(f, &nreq, 8) || nreq > (1u << 20)) return 15;
    const size_t dim = (size_t)1 << n;
    uint8_t *req = (uint8_t *)calloc(nreq ? nreq : 1, 1);
    double *grads = (double *)calloc(nreq ? nreq : 1, sizeof(double));
    arcqml_c128 *psi = (arcqml_c128 *)malloc(dim * sizeof(arcqml_c128));
    arcqml_c128 *lam = (arcqml_c128 *)malloc(dim * sizeof(arcqml_c128));
    arcqml_c128 *scratch = (arcqml_c128 *)malloc(dim * sizeof(arcqml_c128));
    if (!req || !grads || !psi || !lam || !scratch) return 16;
    if (rd(f, req, nreq) || rd(f, &upstream, 8) || rd(f, psi, dim * sizeof(arcqml_c128)) ||
        rd(f, lam, dim * sizeof(arcqml_c128)))
        return 17;
    fclose(f);
    FILE *o = fopen(out_path, "wb");
    if (!o) return 18;
    if (arcqml_rt_v1_circuit_plan_apply(&plan, psi, dim, n) != 0) {
        last_error("circuit_plan_apply");
        return 19;
    }
    fwrite(psi, sizeof(arcqml_c128), dim, o);
    if (arcqml_rt_v1_adjoint_backward(&plan, psi, lam, dim, scratch, n, upstream, req, nreq, grads,
                                      nreq) != 0) {
        last_error("adjoint_backward");
        return 20;
    }
    fwrite(psi, sizeof(arcqml_c128), dim, o);
    fwrite(lam, sizeof(arcqml_c128), dim, o);
    fwrite(grads, sizeof(double), nreq, o);
    fclose(o);
    arcqml_rt_v1_circuit_plan_destroy(&plan);
    free(req);
    free(grads);
    free(psi);
    free(lam);
    free(scratch);
    return 0;
}

int main(int argc, char **argv) {
    if (argc == 2 && strcmp(argv[1], "check") == 0) return check();
    if (argc == 4 && strcmp(argv[1], "run") == 0) return run(argv[2], argv[3]);
    fprintf(stderr, "usage: link_consumer check | run <input> <output>\n");
    return 1;
}
