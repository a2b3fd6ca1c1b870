// kernels/lib.ts drop-in: the reference module's exports over libflock_cuda.so.
//
// What changes for a caller: `getDevice()` resolves to a CudaDevice (one CUDA
// device opened through the C ABI) instead of a WebGPU GPUDevice, and
// `storageBuffer` / `uniformBuffer` / `readBack` move bytes through a
// DeviceBuffer (a flock_tensor holding raw bytes) instead of a GPUBuffer.
// Everything else keeps the reference's names, argument meaning and results:
//   * splitQ8 / splitQ4 call flock_repack_q8/q4 (byte-identical to lib.ts:126,
//     :142);
//   * quantRowQ8/Q4 and quantMatrixQ8/Q4 call flock_quant_q8/q4 (byte-identical
//     to lib.ts:40, :64, :94, :103);
//   * fma32, halfToF32, cpuMatmulQ8F32 / cpuMatmulQ4F32 with SERIAL or coop(n),
//     maxRelErr, randVec, ok and summary are the CPU references the tests
//     compare with, restated here in plain TypeScript (lib.ts:30, :169-318,
//     :322, :595-615): f32 rounding is Math.fround on f64 numbers, exactly
//     the reference's arithmetic.
import { check, flock, FLOCK_E_ARG, FlockError, handleSlot, slotPointer } from "./cuda_ffi.ts";

export const Q8_BLOCK = 32;
export const Q8_BYTES = 34; // f16 scale + 32 int8
export const Q4_BLOCK = 32;
export const Q4_BYTES = 18; // f16 scale + 16 nibble pairs

const fr = Math.fround;

// ------------------------------------------------------------------ device

/**
 * A device-resident hidden-state port of a layer (Layer.inputBuffer() /
 * outputBuffer(); both name the layer's one activation buffer, which the
 * layer updates in place) or one of its caches (cacheBuffers()).
 */
export interface LayerPort {
  readonly layer: EncodableLayer;
  readonly which: "input" | "output" | "k" | "v";
}

/** What the encoder needs from a layer (layer.ts implements it). */
export interface EncodableLayer {
  readonly handle: Deno.PointerValue;
  readonly hidden: number;
  readonly nKeys: number;
  /** flock_layer_encode now: `hidden` null = the input already on the device. */
  runNow(n: number, hidden: Float32Array | null): void;
  readOutputNow(n: number): Float32Array;
  readCacheNow(): { k: Float32Array; v: Float32Array };
}

type Step =
  | { kind: "layer"; layer: EncodableLayer; n: number; hidden: Float32Array | null }
  | { kind: "copy"; src: LayerPort | DeviceBuffer; dst: LayerPort | DeviceBuffer; bytes: number }
  | { kind: "call"; run: () => void };

/**
 * The shim's GPUCommandEncoder: it records layer encodes, buffer copies and
 * sharded-matvec runs, and runs them in order on queue.submit.  A chain
 * "layer(x) -> copy(out, next.in) -> next() -> ..." becomes one
 * flock_range_forward call (the layers run back to back on the device, the
 * hidden state never leaves it), which is what web/bird.html builds with a
 * raw encoder.
 */
export class CommandEncoder {
  readonly steps: Step[] = [];

  /** Called by Layer.encode / encodePrefill with an encoder. */
  pushLayer(layer: EncodableLayer, n: number, hidden: Float32Array | null): void {
    this.steps.push({ kind: "layer", layer, n, hidden });
  }

  /** Called by ShardedMatvec / ShardedHead encode. */
  pushCall(run: () => void): void {
    this.steps.push({ kind: "call", run });
  }

  copyBufferToBuffer(
    src: LayerPort | DeviceBuffer,
    _srcOffset: number,
    dst: LayerPort | DeviceBuffer,
    _dstOffset: number,
    bytes: number,
  ): void {
    this.steps.push({ kind: "copy", src, dst, bytes });
  }

  finish(): CommandBuffer {
    return { steps: this.steps.slice() };
  }
}

export interface CommandBuffer {
  readonly steps: Step[];
}

function isPort(x: LayerPort | DeviceBuffer): x is LayerPort {
  return (x as LayerPort).layer !== undefined;
}

function runSteps(steps: Step[]): void {
  let i = 0;
  while (i < steps.length) {
    const s = steps[i];
    if (s.kind === "call") {
      s.run();
      i++;
      continue;
    }
    if (s.kind === "copy") {
      // a copy that does not chain two layer encodes: through the host
      if (isPort(s.src) && isPort(s.dst) && s.src.which === "output" && s.dst.which === "input") {
        const n = s.bytes / 4 / s.src.layer.hidden;
        const next = steps[i + 1];
        if (next?.kind === "layer" && next.layer === s.dst.layer && next.hidden === null) {
          next.hidden = s.src.layer.readOutputNow(n);
        }
      }
      i++;
      continue;
    }
    // a layer step: extend it over "copy(out -> next.in), next(null)" pairs
    const chain: EncodableLayer[] = [s.layer];
    let j = i + 1;
    while (j + 1 < steps.length) {
      const c = steps[j], l = steps[j + 1];
      if (
        c.kind !== "copy" || l.kind !== "layer" || l.hidden !== null || l.n !== s.n ||
        !isPort(c.src) || !isPort(c.dst) || c.src.layer !== chain[chain.length - 1] ||
        c.dst.layer !== l.layer
      ) break;
      chain.push(l.layer);
      j += 2;
    }
    if (chain.length === 1 || s.hidden === null) {
      s.layer.runNow(s.n, s.hidden);
      i++;
      continue;
    }
    const handles = BigUint64Array.from(
      chain.map((l) => BigInt(Deno.UnsafePointer.value(l.handle))),
    );
    const out = new Float32Array(s.n * s.layer.hidden);
    check(flock().flock_range_forward(handles, chain.length, s.hidden, s.n, s.layer.nKeys, 0, out));
    i = j;
  }
}

/** One CUDA device opened through the C ABI (flock_dev_open). */
export class CudaDevice {
  private constructor(readonly ordinal: number, readonly handle: Deno.PointerValue) {}

  /** GPUDevice.queue.submit: run the recorded steps in order. */
  readonly queue = {
    submit(cmds: CommandBuffer[]): void {
      for (const c of cmds) runSteps(c.steps);
    },
  };

  createCommandEncoder(): CommandEncoder {
    return new CommandEncoder();
  }

  static open(ordinal = 0): CudaDevice {
    const slot = handleSlot();
    check(flock().flock_dev_open(ordinal, slot));
    return new CudaDevice(ordinal, slotPointer(slot));
  }

  /** Wait for every launch this device's stream has queued. */
  sync(): void {
    check(flock().flock_dev_sync(this.handle));
  }

  smCount(): number {
    const n = new Int32Array(1);
    check(flock().flock_dev_sm_count(this.handle, n));
    return n[0];
  }

  close(): void {
    check(flock().flock_dev_close(this.handle));
  }
}

/**
 * lib.ts:385 getDevice: the device the kernels run on.  The reference raises
 * WebGPU's buffer-binding limits; a CUDA device has no binding limit, so the
 * only choice left is the ordinal (FLOCK_DEVICE, default 0).
 */
export function getDevice(ordinal?: number): Promise<CudaDevice> {
  const o = ordinal ?? Number(Deno.env.get("FLOCK_DEVICE") ?? "0");
  return Promise.resolve(CudaDevice.open(o));
}

/** Raw bytes resident on a device: the shim's GPUBuffer. */
export class DeviceBuffer {
  constructor(
    readonly dev: CudaDevice,
    readonly handle: Deno.PointerValue,
    readonly size: number,
  ) {}

  destroy(): void {
    check(flock().flock_tensor_free(this.handle));
  }
}

function asBytes(data: Uint8Array | Float32Array | Uint32Array): Uint8Array {
  return data instanceof Uint8Array
    ? data
    : new Uint8Array(data.buffer, data.byteOffset, data.byteLength);
}

/** lib.ts:548 storageBuffer: upload `data` (size rounded up to 4 bytes). */
export function storageBuffer(dev: CudaDevice, data: Uint8Array | Float32Array): DeviceBuffer {
  const bytes = asBytes(data);
  const slot = handleSlot();
  check(flock().flock_tensor_from_bytes(dev.handle, bytes, bytes.byteLength, slot));
  return new DeviceBuffer(dev, slotPointer(slot), (bytes.byteLength + 3) & ~3);
}

/** lib.ts:569 uniformBuffer: u32 values, padded to 16 bytes as WebGPU pads. */
export function uniformBuffer(dev: CudaDevice, vals: number[]): DeviceBuffer {
  const size = Math.max(16, (vals.length * 4 + 15) & ~15);
  const words = new Uint32Array(size / 4);
  words.set(vals);
  return storageBuffer(dev, new Uint8Array(words.buffer));
}

/** lib.ts:576 readBack: the first `bytes` of `src` as f32 (a raw buffer, a
 *  layer's hidden state, or its K/V cache). */
export function readBack(
  _dev: CudaDevice,
  src: DeviceBuffer | LayerPort,
  bytes: number,
): Promise<Float32Array> {
  const n = Math.ceil(bytes / 4);
  if (isPort(src)) {
    if (src.which === "k" || src.which === "v") {
      return Promise.resolve(src.layer.readCacheNow()[src.which].slice(0, n));
    }
    const rows = Math.max(1, Math.ceil(n / src.layer.hidden));
    return Promise.resolve(src.layer.readOutputNow(rows).slice(0, n));
  }
  const out = new Float32Array(n);
  check(flock().flock_tensor_read(src.handle, 0, bytes, new Uint8Array(out.buffer)));
  return Promise.resolve(out);
}

// ------------------------------------------------------------ quantizing

/** lib.ts:30 halfToF32 (inf widens to the largest finite f32, as the kernels clamp). */
export function halfToF32(h: number): number {
  const sign = h & 0x8000 ? -1 : 1;
  const e = (h >> 10) & 31, m = h & 1023;
  if (e === 31) return sign * 3.4028235e38;
  if (e === 0) return sign * m * 2 ** -24;
  return sign * (1024 + m) * 2 ** (e - 25);
}

function quantize(kind: "q8" | "q4", w: Float32Array, rows: number, cols: number): Uint8Array {
  if (cols % 32 !== 0 || w.length !== rows * cols) {
    throw new FlockError(FLOCK_E_ARG, `quantize: ${rows}x${cols} does not fit ${w.length} values`);
  }
  const out = new Uint8Array((rows * cols / 32) * (kind === "q8" ? Q8_BYTES : Q4_BYTES));
  const f = kind === "q8" ? flock().flock_quant_q8 : flock().flock_quant_q4;
  check(f(new Uint8Array(w.buffer, w.byteOffset, w.byteLength), rows, cols, out));
  return out;
}

/** lib.ts:40 quantRowQ8. */
export function quantRowQ8(vals: Float32Array): Uint8Array {
  return quantize("q8", vals, 1, vals.length);
}

/** lib.ts:64 quantRowQ4 (ggml nibble order: byte i = q[i] | q[i+16] << 4). */
export function quantRowQ4(vals: Float32Array): Uint8Array {
  return quantize("q4", vals, 1, vals.length);
}

/** lib.ts:94 quantMatrixQ8. */
export function quantMatrixQ8(w: Float32Array, rows: number, cols: number): Uint8Array {
  return quantize("q8", w, rows, cols);
}

/** lib.ts:103 quantMatrixQ4. */
export function quantMatrixQ4(w: Float32Array, rows: number, cols: number): Uint8Array {
  return quantize("q4", w, rows, cols);
}

// -------------------------------------------------------------- repacking

export interface SplitQ8 {
  qs: Uint8Array;
  scales: Uint8Array;
}

function split(kind: "q8" | "q4", packed: Uint8Array, rows: number, cols: number): SplitQ8 {
  const blocks = rows * (cols / 32);
  const qs = new Uint8Array(kind === "q8" ? rows * cols : blocks * 16);
  const scales = new Uint8Array(blocks * 2);
  const f = kind === "q8" ? flock().flock_repack_q8 : flock().flock_repack_q4;
  check(f(packed, rows, cols, qs, scales));
  return { qs, scales };
}

/** lib.ts:126 splitQ8: 34-byte blocks -> contiguous int8 plane + f16 scale plane. */
export function splitQ8(packed: Uint8Array, rows: number, cols: number): SplitQ8 {
  return split("q8", packed, rows, cols);
}

/** lib.ts:142 splitQ4: 18-byte blocks -> nibble plane + f16 scale plane. */
export function splitQ4(packed: Uint8Array, rows: number, cols: number): SplitQ8 {
  return split("q4", packed, rows, cols);
}

// ---------------------------------------------------- CPU references (tests)

/** lib.ts:169 fma32: the f64 product is exact, the add and the f32 cast round. */
export function fma32(a: number, b: number, c: number): number {
  return fr(a * b + c);
}

export type Reduction = { kind: "serial" } | { kind: "coop"; lanes: number };
export const SERIAL: Reduction = { kind: "serial" };
export const coop = (lanes: number): Reduction => ({ kind: "coop", lanes });

type Block = { scale: number; q: Int8Array };

function q8Block(p: Uint8Array, at: number): Block {
  const q = new Int8Array(32);
  for (let i = 0; i < 32; i++) q[i] = (p[at + 2 + i] << 24) >> 24;
  return { scale: fr(halfToF32(p[at] | (p[at + 1] << 8))), q };
}

function q4Block(p: Uint8Array, at: number): Block {
  const q = new Int8Array(32);
  for (let i = 0; i < 16; i++) {
    q[i] = (p[at + 2 + i] & 15) - 8;
    q[i + 16] = (p[at + 2 + i] >> 4) - 8;
  }
  return { scale: fr(halfToF32(p[at] | (p[at + 1] << 8))), q };
}

// dot of four quants with four inputs: the first product rounded, then three fma32
function dot4(q: Int8Array, x: Float32Array, qi: number[], xo: number): number {
  let s = fr(q[qi[0]] * x[xo + qi[0]]);
  for (let k = 1; k < 4; k++) s = fma32(q[qi[k]], x[xo + qi[k]], s);
  return s;
}

function treeSum(v: Float32Array): number {
  const b = Float32Array.from(v);
  for (let half = b.length >> 1; half > 0; half >>= 1) {
    for (let i = 0; i < half; i++) b[i] = fr(b[i] + b[i + half]);
  }
  return b[0];
}

/**
 * lib.ts:213 matmulF32: y[r] = sum over 32-weight blocks of scale * dot.
 * SERIAL folds the 32 products of a block with fma32 in order.  coop(n) gives
 * block b to lane b % n; per block four (lo, hi) quads are each dot4'd, their
 * sum rounded, and folded into the lane with fma32(scale, ., lane); the n lanes
 * are tree-summed.  `quads` are the weight indices of the four quad pairs.
 */
function blockMatmul(
  packed: Uint8Array,
  x: Float32Array,
  rows: number,
  cols: number,
  red: Reduction,
  blockBytes: number,
  decode: (p: Uint8Array, at: number) => Block,
  quads: [number[], number[]][],
): Float32Array {
  const nb = cols / 32;
  const y = new Float32Array(rows);
  const lanes = new Float32Array(red.kind === "coop" ? red.lanes : 1);
  for (let r = 0; r < rows; r++) {
    lanes.fill(0);
    for (let b = 0; b < nb; b++) {
      const { scale, q } = decode(packed, (r * nb + b) * blockBytes);
      if (red.kind === "serial") {
        let s = 0;
        for (let i = 0; i < 32; i++) s = fma32(q[i], x[b * 32 + i], s);
        lanes[0] = fma32(scale, s, lanes[0]);
        continue;
      }
      const l = b % red.lanes;
      for (const [lo, hi] of quads) {
        const d = fr(dot4(q, x, lo, b * 32) + dot4(q, x, hi, b * 32));
        lanes[l] = fma32(scale, d, lanes[l]);
      }
    }
    y[r] = red.kind === "serial" ? lanes[0] : treeSum(lanes);
  }
  return y;
}

const range4 = (base: number) => [base, base + 1, base + 2, base + 3];

/** lib.ts:251 cpuMatmulQ8F32: quads (8g..8g+3, 8g+4..8g+7). */
export function cpuMatmulQ8F32(
  packed: Uint8Array,
  x: Float32Array,
  rows: number,
  cols: number,
  red: Reduction = SERIAL,
): Float32Array {
  const quads = [0, 1, 2, 3].map((g) => [range4(8 * g), range4(8 * g + 4)] as [number[], number[]]);
  return blockMatmul(packed, x, rows, cols, red, Q8_BYTES, q8Block, quads);
}

/** lib.ts:280 cpuMatmulQ4F32: quads (4g..4g+3, 16+4g..16+4g+3), nibble order. */
export function cpuMatmulQ4F32(
  packed: Uint8Array,
  x: Float32Array,
  rows: number,
  cols: number,
  red: Reduction = SERIAL,
): Float32Array {
  const quads = [0, 1, 2, 3].map((g) => [range4(4 * g), range4(16 + 4 * g)] as [number[], number[]]);
  return blockMatmul(packed, x, rows, cols, red, Q4_BYTES, q4Block, quads);
}

/** lib.ts:322 maxRelErr with the 1e-6 denominator floor. */
export function maxRelErr(a: Float32Array, b: Float32Array): number {
  let worst = 0;
  for (let i = 0; i < a.length; i++) {
    worst = Math.max(worst, Math.abs(a[i] - b[i]) / Math.max(1e-6, Math.abs(b[i])));
  }
  return worst;
}

/** lib.ts:595 randVec: uniform in [-scale, scale). */
export function randVec(n: number, scale = 1): Float32Array {
  const v = new Float32Array(n);
  for (let i = 0; i < n; i++) v[i] = (2 * Math.random() - 1) * scale;
  return v;
}

let passed = 0, failed = 0;

/** lib.ts:604 ok: one reported check. */
export function ok(name: string, cond: boolean, extra = ""): void {
  if (cond) passed++;
  else failed++;
  console.log(`  ${cond ? "ok  " : "FAIL"} ${name}${extra ? "  " + extra : ""}`);
}

/** lib.ts:613 summary: prints the tally, returns the failure count. */
export function summary(): number {
  console.log(`\n${passed} passed, ${failed} failed`);
  return failed;
}
