/*
 * candelora_iq2_testing.h -- test hooks of libcandelora_iq2.so. Not for production use: they exist
 * so that the failure-detection paths of the library can be exercised without faulting a GPU.
 * No counterpart in the reference (its Metal kernels have no bounded waits).
 */
#ifndef CANDELORA_IQ2_TESTING_H
#define CANDELORA_IQ2_TESTING_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Process-wide, for later prefill-GEMM launches (m > 32): the bound of every pipeline wait
 * (wait_limit_ns; 0 restores the default 2 s) and, when stall_stage > 0, a stage (1-based) of
 * every CTA whose "weights written" arrival the decode warps withhold. The MMA thread's wait on
 * that stage then runs out after wait_limit_ns (a flag that nothing sets): the kernel records the
 * timeout in the device status that iq2_device_check reports, stops issuing work, waits (bounded)
 * for what it already issued and frees its tensor memory. stall_stage = 0 restores normal runs.
 */
int iq2_testing_set_gemm_stall(uint64_t wait_limit_ns, uint32_t stall_stage);

#ifdef __cplusplus
}
#endif

#endif /* CANDELORA_IQ2_TESTING_H */
