// ne_fault.h -- host-side fault injection points (fault.cu).
#pragma once

#include "../../include/ne.h"

namespace ne {

// True when NE_FAULT_INJECT makes this call of `entry` fail; *status then
// holds the status to return.  Counts the call either way (entries that no
// item names cost one branch).
bool fault_point(const char* entry, ne_status* status);

}  // namespace ne

// At the top of a C-ABI entry point that takes a context (after its argument
// checks; needs ne_ctx.h's fail): an injected failure returns with
// ne_last_error naming it.
#define NE_FAULT_POINT(ctx, name)                                                        \
  do {                                                                                   \
    ne_status fs_;                                                                       \
    if (::ne::fault_point(name, &fs_))                                                   \
      return ::ne::fail((ctx), fs_, "injected fault (NE_FAULT_INJECT " name ")");         \
  } while (0)
