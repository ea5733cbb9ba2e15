// The public entry points of wgblas (the reference's index.mjs) for the
// sgemm/dgemm path: the same names and argument orders, backed by the CUDA
// library through the Node-API addon (../wgblas_napi.c).
export { init, cleanup, gpuName } from "./src/init.mjs";
export { sgemm } from "./src/sgemm/sgemm.mjs";
export { dgemm } from "./src/dgemm/dgemm.mjs";
export { GpuMatrix } from "./src/classes/GpuMatrix.mjs";
export { GpuVector } from "./src/classes/GpuVector.mjs";
export { randomFloat32Array, randomFloat64Array } from "./src/random/random.mjs";
export { sgemmSharded, dgemmSharded, commUniqueId, Comm } from "./src/shard.mjs";
