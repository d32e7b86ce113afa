// Single translation unit of libyolob200.so: device globals shared by the kernels (the
// device error word) then need no relocatable device code.
#include "conv_misc.cu"
#include "conv_tc.cu"
#include "conv_pair.cu"
#include "conv_patch.cu"
#include "conv_kxn.cu"
#include "attn.cu"
#include "post.cu"
#include "cls.cu"
#include "obb.cu"
#include "engine.cu"
