// Device-only translation unit: the KV-cache entries as a cubin (glm_glue_b200.cubin) exposing the
// kern-glm53 glue entry names and parameter lists, for a kern manifest. Launch shapes are listed
// beside each entry in glmkv_kernels.cuh.
#include "glmkv_kernels.cuh"
#include "glmkv_mqa.cuh"
