// kernels/shard.ts drop-in: ShardedMatvec and ShardedHead on CUDA through
// libflock_cuda.so.  All shards live on one device, as in the reference's
// single-device validation form; "row" shards concatenate bit-identically,
// "col" shards sum their partials in shard order (shardReduceRef), and the
// head reduces per-shard argmaxes by reduceShardArgmax's tie rule.  The
// shard ranges are the reference's own shardRanges (shard_ref.ts:97), and the
// binding-limit error is the C ABI's FLOCK_E_LIMIT with the reference's text
// (shard.ts:229-243).
//
// One difference a caller can see: a run computes the shards and the reduce
// together, so encodeShardsOnly() records the whole run and
// encodeReduceOnly() / dispatchReduce() record nothing.
import { check, flock, handleSlot, slotPointer } from "./cuda_ffi.ts";
import { type CommandEncoder, type CudaDevice, type SplitQ8 } from "./lib.ts";
import { type ShardRange, shardRanges } from "./shard_ref.ts";

export type Direction = "row" | "col";

/** shard.ts:104 ShardedMatvecOpts. */
export interface ShardedMatvecOpts {
  /** Largest byte size one shard's weight binding may have (none if omitted). */
  bindingLimit?: number;
}

/** The host-side result of the last run, read through output() / logits(). */
export class HostResult {
  data: Float32Array;
  constructor(n: number) {
    this.data = new Float32Array(n);
  }
}

/** shard.ts:138 ShardedMatvec. */
export class ShardedMatvec {
  readonly ranges: ShardRange[];
  readonly uploadedBytes: number;
  private x: Float32Array;
  private readonly out: HostResult;
  private freed = false;

  private constructor(
    readonly rows: number,
    readonly cols: number,
    readonly direction: Direction,
    n: number,
    readonly handle: Deno.PointerValue,
  ) {
    this.ranges = shardRanges(direction === "row" ? rows : cols, n, direction === "row" ? 1 : 32);
    this.uploadedBytes = rows * cols + (rows * cols / 32) * 2;
    this.x = new Float32Array(cols);
    this.out = new HostResult(rows);
  }

  /** shard.ts:214 create(dev, split, rows, cols, n, direction, opts). */
  static create(
    dev: CudaDevice,
    split: SplitQ8,
    rows: number,
    cols: number,
    n: number,
    direction: Direction,
    opts: ShardedMatvecOpts = {},
  ): Promise<ShardedMatvec> {
    const slot = handleSlot();
    check(flock().flock_shard_matvec_create(dev.handle, split.qs, split.scales, rows, cols, n,
      direction === "row" ? 0 : 1, opts.bindingLimit ?? -1, slot));
    return Promise.resolve(new ShardedMatvec(rows, cols, direction, n, slotPointer(slot)));
  }

  /** shard.ts:320 setInput. */
  setInput(x: Float32Array): void {
    if (x.length !== this.cols) throw new Error(`input has ${x.length} values, expected ${this.cols}`);
    this.x = Float32Array.from(x);
  }

  private run(): void {
    check(flock().flock_shard_matvec_run(this.handle, this.x, this.out.data));
  }

  /** shard.ts:340 encode: the shards and (col) the reduce. */
  encode(enc: CommandEncoder): void {
    enc.pushCall(() => this.run());
  }

  /** shard.ts:352 encodeShardsOnly: the whole run (see the header). */
  encodeShardsOnly(enc: CommandEncoder): void {
    enc.pushCall(() => this.run());
  }

  /** shard.ts:359 encodeReduceOnly: nothing left to record. */
  encodeReduceOnly(_enc: CommandEncoder): void {}

  /** shard.ts:383 dispatchShards: run now. */
  dispatchShards(_p?: unknown): void {
    this.run();
  }

  /** shard.ts:392 dispatchReduce: the reduce ran with the shards. */
  dispatchReduce(_p?: unknown): void {}

  /** shard.ts:400 output: y = W x of the last run. */
  output(): HostResult {
    return this.out;
  }

  /** shard.ts:405 partials: [n][rows] per-shard products ("col" only). */
  partials(): Float32Array {
    const p = new Float32Array(this.ranges.length * this.rows);
    check(flock().flock_shard_matvec_partials(this.handle, p));
    return p;
  }

  /** shard.ts:411 wireBytesPerCall: the bytes a multi-device run would move. */
  wireBytesPerCall(): number {
    const n = new BigInt64Array(1);
    check(flock().flock_shard_matvec_wire_bytes(this.handle, n));
    return Number(n[0]);
  }

  /** shard.ts:421 destroy. */
  destroy(): void {
    if (this.freed) return;
    this.freed = true;
    check(flock().flock_shard_matvec_free(this.handle));
  }
}

/** shard.ts:440 ShardedHeadOpts. */
export interface ShardedHeadOpts extends ShardedMatvecOpts {
  shards: number;
}

/** shard.ts:459 ShardedHead: the row-sharded LM head with the sharded argmax. */
export class ShardedHead {
  readonly nShards: number;
  private x: Float32Array;
  private readonly out: HostResult;
  private token = -1;
  private readonly ranges: ShardRange[];
  private freed = false;

  private constructor(
    readonly vocab: number,
    readonly hidden: number,
    shards: number,
    readonly handle: Deno.PointerValue,
  ) {
    this.nShards = shards;
    this.ranges = shardRanges(vocab, shards, 1);
    this.x = new Float32Array(hidden);
    this.out = new HostResult(vocab);
  }

  /** shard.ts:502 create(dev, split, vocab, hidden, {shards}). */
  static create(
    dev: CudaDevice,
    split: SplitQ8,
    vocab: number,
    hidden: number,
    opts: ShardedHeadOpts,
  ): Promise<ShardedHead> {
    const slot = handleSlot();
    check(flock().flock_sharded_head_create(dev.handle, split.qs, split.scales, vocab, hidden,
      opts.shards, slot));
    return Promise.resolve(new ShardedHead(vocab, hidden, opts.shards, slotPointer(slot)));
  }

  /** shard.ts:582 setInput: the normed hidden state. */
  setInput(h: Float32Array): void {
    if (h.length !== this.hidden) throw new Error(`input has ${h.length} values, expected ${this.hidden}`);
    this.x = Float32Array.from(h);
  }

  /** shard.ts:595 encode: logits, per-shard argmax, cross-shard reduce. */
  encode(enc: CommandEncoder): void {
    enc.pushCall(() => {
      const t = new Int32Array(1);
      check(flock().flock_sharded_head_run(this.handle, this.x, this.out.data, t));
      this.token = t[0];
    });
  }

  /** shard.ts:627 logits: [vocab] of the last run. */
  logits(): HostResult {
    return this.out;
  }

  /** The id the cross-shard reduce chose in the last run. */
  chosen(): number {
    return this.token;
  }

  /** shard.ts:632 argmaxBuffers: per shard (value, local index, row offset). */
  argmaxBuffers(): { oVal: Float32Array; oIdx: Uint32Array; rowOffset: number }[] {
    const n = this.nShards;
    const vals = new Float32Array(n), idx = new BigInt64Array(n), off = new BigInt64Array(n);
    check(flock().flock_sharded_head_shard_argmax(this.handle, vals, idx, off));
    return Array.from({ length: n }, (_, s) => ({
      oVal: Float32Array.of(vals[s]),
      oIdx: Uint32Array.of(Number(idx[s])),
      rowOffset: Number(off[s]),
    }));
  }

  /** shard.ts:641 shardBytes: Q8_0 bytes each shard holds (qs + scales). */
  shardBytes(): number[] {
    return this.ranges.map((r) => r.count * this.hidden + (r.count * this.hidden / 32) * 2);
  }

  /** shard.ts:645 destroy. */
  destroy(): void {
    if (this.freed) return;
    this.freed = true;
    check(flock().flock_sharded_head_free(this.handle));
  }
}
