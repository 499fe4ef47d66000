// The persistent step kernel's split-replay instantiations (replay mode, no flush,
// T and c also written to the caller's buffers; gdnr_replay_split), in a module
// of their own: see launch_step5_split in gdnr_step5.cu.
#define GDNR_S5_SPLIT_TU
#include "gdnr_step5.cu"
