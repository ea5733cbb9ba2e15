// Seeded inputs (src/random/random.mjs:14-26): mulberry32 draws u in [0, 1),
// value = low + u*(high-low); with a seed the arrays match the reference's.
// Without one the seed comes from Math.random, as the reference's unseeded calls
// are random too.
import { addon } from "../addon.mjs";

function seedOf(seed) {
  return seed === undefined ? Math.floor(Math.random() * 2 ** 32) : seed >>> 0;
}

export function randomFloat32Array(n, low = -1, high = 1, seed = undefined) {
  return addon.randomArray(n, low, high, seedOf(seed), false);
}

export function randomFloat64Array(n, low = -1, high = 1, seed = undefined) {
  return addon.randomArray(n, low, high, seedOf(seed), true);
}
