/*
 * Extensions of the armcc SDK session API (armcc_sdk.h) provided by
 * libsg_b200.so.  No reference counterpart.
 */
#ifndef SG_SDK_EXT_H_
#define SG_SDK_EXT_H_

#include "armcc_sdk.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Copies the fp32 logits of the last processed token (after
 * armsess_prefill, or after a armsess_decode that ran a step) into host
 * memory: min(n, vocab) values.  Returns ARMCC_OK, or an error status with
 * armpack_last_error() set. */
ArmStatus sg_session_last_logits(ArmSession* sess, float* host_out, uint32_t n);

/* Number of tokens in the session's KV cache. */
uint32_t sg_session_position(const ArmSession* sess);

#ifdef __cplusplus
}
#endif
#endif /* SG_SDK_EXT_H_ */
