// The tensor-parallel instance of the persistent decode kernel
// (k_decode_persistent<true>) in its own translation unit: persist.cu compiled
// again with QB_PERSIST_TP, which keeps its device code and emits only this
// instance and its launcher (launch_persistent_tp), so that the single-GPU
// module holds none of the exchange paths.
#define QB_PERSIST_TP 1
#include "persist.cu"
