// The fused decode kernel (decode_fused.cu) compiled for a group of GPUs
// (tmg_fused_group_init): one joint grid over the ranks' SMs for the GEMV
// phases, every exchanged word, KV append and argmax candidate stored into
// every rank's memory over NVLink (system-scope stores), polls of the local
// copies at system scope; each rank runs every attention item itself.
// A separate translation unit so that the single-GPU kernels keep none of
// these branches.
#define TMG_FUSED_GROUP 1
#include "decode_fused.cu"
