// Loads the Node-API addon (wgblas_napi.node, built next to libwgblas_b200.so by
// wgblas_b200/build.py). WGBLAS_NAPI_ADDON names another build. Loading fails
// loudly: there is no CPU fallback.
import { createRequire } from "node:module";
import { fileURLToPath } from "node:url";
import path from "node:path";

const here = path.dirname(fileURLToPath(import.meta.url));
const require = createRequire(import.meta.url);
const file = process.env.WGBLAS_NAPI_ADDON || path.join(here, "..", "..", "wgblas_napi.node");

export const addon = require(file);
