// kernels_f16h.cu — kernel instantiations for FP16 values summed in FP16 (half16).
#define VALUE_TYPE half16
#define LAUNCH_TILES_NAME launch_tiles_f16h
#define LAUNCH_VECTOR_NAME launch_vector_f16h
#define TILES_OCCUPANCY_NAME tiles_occupancy_f16h
#define LAUNCH_CLASSES_NAME launch_classes_f16h
#define PREPARE_CLASSES_NAME prepare_classes_f16h
#include "kernels_instantiate.cuh"
