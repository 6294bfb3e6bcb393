// The communicator handle of the C ABI (runtime.cu), shared with the ResNet
// step, whose data-parallel communicator is exposed through the same handle.
#pragma once

#include <nccl.h>

struct rnn_comm {
  ncclComm_t comm = nullptr;
  int device = 0, rank = 0, world = 1;
  bool aborted = false;  // ncclCommAbort ran: the communicator is gone
  bool owned = true;     // false: borrowed from a network, which destroys it
};
