/*
 * msda_b200_checked.h -- the one extra entry point of the checked build of
 * libmsda_b200.so (msda_triton_b200/_lib_checked/, compiled with
 * -DMSDA_CHECKED by `python -m msda_triton_b200.build --checked`).
 *
 * The checked build runs the same kernels with a bounds check on every value
 * gather and value-gradient scatter: an address outside its buffer is not
 * accessed and sets a bit of a per-device word (1: value gather, 2: 16-bit
 * grad_value scatter, 4: fp32 accumulator scatter, 8: a kernel whose
 * shared-memory layout would pass its launch's size and which therefore did
 * no work).  It stands in for a
 * memory checker and is for tests and debugging; it is slower.  In the
 * cell-sorted backward the value gathers are checked; its record, fp32
 * accumulator and grad_value stores are not instrumented.
 */
#ifndef MSDA_B200_CHECKED_H_
#define MSDA_B200_CHECKED_H_

#include "msda_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Bits recorded on the current device since the last clear (0: no
 * violation; 0xffffffff: the word could not be read).  Synchronises the
 * device; `clear` != 0 resets the word. */
MSDA_API unsigned int msda_checked_violations(int clear);

#ifdef __cplusplus
}
#endif

#endif /* MSDA_B200_CHECKED_H_ */
