// The generic decode path (decode_generic.cu) as seen from the launchers in decode.cu.
#pragma once

#include <stddef.h>

#include "../../include/flashspec_b200.h"

namespace fsb {

// True when the generic kernel handles these arguments (head_dim 32/64/128/256, quant
// block <= 64 tokens, page a multiple of the quant block, fp16/bf16 q, <= 8 q heads per
// kv head).
bool generic_supports(const FsDecodeArgs* a);
// Workspace bytes of a generic call (its split partials) and the split count used.
size_t generic_workspace(const FsDecodeArgs* a, int device, int* splits_out);
int launch_generic_decode(const FsDecodeArgs* a, int device, void* stream);

}  // namespace fsb
