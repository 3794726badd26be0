// module.cu - builds cudair_kernels.cubin: the loadable sm_100a module whose
// entry points keep the reference's kernel names and parameter ABI
// (MatMul16, VecAdd, ReduceF32, and the rest of the reference's vecadd and
// hopper example packages).  A caller loads it with cuModuleLoadData
// (gocudrv ctx.LoadModule, or cudair_module_load) exactly where the
// reference loads the PTX its compiler produced (main_test.go:187).
#include "module_kernels.cuh"
#include "module_demos.cuh"
