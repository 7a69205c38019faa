// Unity build of libqqt_b200.so: one translation unit so the device error
// word and helpers are shared without relocatable device code.
#include "sim_observe.cu"
#include "sim_step.cu"
#include "sim_reset.cu"
#include "policy_mlp.cu"
#include "policy_cnn.cu"
#include "train_gae.cu"
#include "train_mlp.cu"
#include "phase_stamps.cu"
