// inference-b200.js -- the B200 stage engine behind the engine contract of
// web/inference-worker.js:13-19 (same exports), for web/tabnet-node.js:19:
//
//   import { initStage, forward, freeStage } from "./inference-b200.js";
//
// The addon (tabnet_b200.c, built by `node-gyp rebuild` in this directory)
// runs every engine call on the libuv thread pool and resolves a Promise.
import { createRequire } from "node:module";

const addon = createRequire(import.meta.url)("./build/Release/tabnet_b200.node");

export async function initStage(spec) { return addon.initStage(spec); }     // -> ctx
export async function forward(ctx, req) { return addon.forward(ctx, req); }  // -> {hidden} | {token_id}
export function freeStage(ctx) { addon.freeStage(ctx); }
export const forwardSafe = forward;
export const forwardLast = forward;
