// kernels_f32.cu — kernel instantiations for float values.
#define VALUE_TYPE float
#define LAUNCH_TILES_NAME launch_tiles_f32
#define LAUNCH_VECTOR_NAME launch_vector_f32
#define TILES_OCCUPANCY_NAME tiles_occupancy_f32
#define LAUNCH_CLASSES_NAME launch_classes_f32
#define PREPARE_CLASSES_NAME prepare_classes_f32
#include "kernels_instantiate.cuh"
