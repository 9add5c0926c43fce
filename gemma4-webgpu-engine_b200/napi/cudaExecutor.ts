// cudaExecutor.ts -- the reference host's ForwardExecutor (src/runtime.ts:73-88) over the
// gemma4_cuda.node addon (g4_napi.c). engine.ts builds a CudaExecutor where it builds GpuExecutor
// today (src/engine.ts:723-761); plan.ts (runGreedyLoop), kv.ts (planKvReuse, KvCacheState) and
// draft.ts (runSpeculativeLoop) stay as they are.
import type { ForwardExecutor } from './runtime';

export interface Gemma4CudaAddon {
  createContext(device: number, options?: Record<string, number | boolean>): unknown;
  destroyContext(ctx: unknown): void;
  initRandom(ctx: unknown, seed: number): void;
  uploadWeight(ctx: unknown, name: string, bytes: Uint8Array, offset: number, total: number): void;
  setScalar(ctx: unknown, name: string, value: number): void;
  prefill(ctx: unknown, seq: number, ids: Int32Array, startPosition: number, isLast: boolean): number;
  decode(ctx: unknown, seq: number, prevToken: number, position: number): number;
  decodeAhead(ctx: unknown, seq: number, position: number): number;
  verify(ctx: unknown, seq: number, tokens: Int32Array, position: number): number[];
  decodeBatch(ctx: unknown, seqs: Int32Array, tokens: Int32Array, positions: Int32Array): number[];
  kvTruncate(ctx: unknown, seq: number, n: number): void;
  readLogits(ctx: unknown, column: number, out: Float32Array): void;
  version(): string;
}

// eslint-disable-next-line @typescript-eslint/no-var-requires
const addon: Gemma4CudaAddon = require('../lib/gemma4_cuda.node');

/**
 * One sequence slot of a CUDA context. Every call is one C-ABI call; the library checks positions
 * against its own KV bookkeeping, so a rewind from planKvReuse also calls kvTruncate.
 */
export class CudaExecutor implements ForwardExecutor {
  constructor(private readonly ctx: unknown, private readonly seq = 0) {}

  static create(device: number, options: Record<string, number | boolean>, seed?: number): CudaExecutor {
    const ctx = addon.createContext(device, options);
    if (seed !== undefined) addon.initRandom(ctx, seed);
    return new CudaExecutor(ctx);
  }

  async prefill(tokens: readonly number[], startPosition: number, isLast: boolean): Promise<number> {
    return addon.prefill(this.ctx, this.seq, Int32Array.from(tokens), startPosition, isLast);
  }

  async decode(prevToken: number, position: number): Promise<number> {
    return addon.decode(this.ctx, this.seq, prevToken, position);
  }

  async decodeAhead(position: number): Promise<number> {
    return addon.decodeAhead(this.ctx, this.seq, position);
  }

  async verify(tokens: readonly number[], position: number): Promise<number[]> {
    return addon.verify(this.ctx, this.seq, Int32Array.from(tokens), position);
  }

  truncate(n: number): void {
    addon.kvTruncate(this.ctx, this.seq, n);
  }

  dispose(): void {
    addon.destroyContext(this.ctx);
  }
}
