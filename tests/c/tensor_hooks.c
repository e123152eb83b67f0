/*
 * tensor_hooks.c - the one library hook sapphire_b200/csrc/tensor.c calls
 * (normally defined in context.cu, where it drops a released tensor's device
 * copies), for host-only builds of the tensor API: tests/test_reference_c.py
 * links the reference's src/test/test_tensor.c against tensor.c with
 * AddressSanitizer and UndefinedBehaviorSanitizer and this file.
 */
#include <stdint.h>

void sapphire_on_tensor_release(uint64_t uid) { (void)uid; }
