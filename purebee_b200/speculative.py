"""Self-speculative decoding (speculative.js:27-204 SelfSpeculativeDecoder).

Drafts `draftCount` tokens with the first `draftLayers` layers, rolls the KV
cache back, verifies each draft with the full model one token at a time,
accepts up to the first mismatch (taking the full model's token there), and
adds a bonus token when every draft was accepted.  The steps are the
runtime's device calls: a layer-limited decode graph for a draft, the full
graph for a verification, the argmax fused into each step's head, and the
cache rollback.  Greedy mode therefore copies one token per step and no
logits; sampling mode draws on the device from the step's logits.

The reference draws with Math.random(); here draw i uses
pb_sample_uniform(seed, i), counting every draw of the generation in order.
"""
from __future__ import annotations

import os
import time
from typing import Optional


class SelfSpeculativeDecoder:
    def __init__(self, runtime, options: Optional[dict] = None):
        options = options or {}
        self.runtime = runtime
        self.draftLayers = options.get("draftLayers") or 4
        self.draftCount = options.get("draftCount") or 4
        self.temperature = options.get("temperature") or 0.6
        self.topK = options.get("topK") or 40
        self._totalRounds = 0
        self._totalDrafted = 0
        self._totalAccepted = 0

    def generate(self, promptTokens, maxTokens: int = 50, opts: Optional[dict] = None):
        """speculative.js:58-189 generate(promptTokens, maxTokens, opts)."""
        opts = opts or {}
        temperature = opts.get("temperature") or self.temperature
        topK = opts.get("topK") or self.topK
        eosIds = opts.get("eosIds") or [2]
        onToken = opts.get("onToken")
        greedy = opts.get("greedy") or False
        seed = opts.get("seed")
        if seed is None:
            seed = int.from_bytes(os.urandom(8), "little")
        rt = self.runtime
        draws = [0]

        def pick(logits_ready_step):
            # the token after the last forward: device argmax, or a device draw
            if greedy:
                return logits_ready_step
            tok = rt.sampleLast(topK, temperature, seed, draws[0])
            draws[0] += 1
            return tok

        rt.resetCache()
        allTokens = list(promptTokens)
        t0 = time.perf_counter()
        out = rt.forward(list(promptTokens), 0)  # prefill
        prefillTime = (time.perf_counter() - t0) * 1000
        pos = len(promptTokens)
        nextToken = rt.argmax(out["logits"]) if greedy else pick(None)
        allTokens.append(nextToken)
        if onToken:
            onToken(nextToken, 0)
        generated = 1
        hitEos = nextToken in eosIds
        d0 = time.perf_counter()

        while generated < maxTokens and not hitEos:
            # draft with the first draftLayers layers
            draftTokens = [nextToken]
            draftPos = pos
            d = 0
            while d < self.draftCount and generated + d < maxTokens:
                current = draftTokens[-1]
                if current in eosIds:
                    break
                g = rt.step(current, draftPos, self.draftLayers)
                draftPos += 1
                draftTokens.append(pick(g))
                d += 1
            numDrafted = len(draftTokens) - 1
            if numDrafted == 0:
                break
            self._totalDrafted += numDrafted
            self._totalRounds += 1
            # verify with the full model, one token at a time
            rt.rollbackCache(pos)
            accepted = 0
            for d in range(numDrafted):
                verifyPred = pick(rt.step(draftTokens[d], pos + d))
                draftPred = draftTokens[d + 1]
                if verifyPred == draftPred:
                    accepted += 1
                    allTokens.append(draftPred)
                    generated += 1
                    if onToken:
                        onToken(draftPred, generated - 1)
                    if draftPred in eosIds:
                        hitEos = True
                        break
                else:
                    allTokens.append(verifyPred)
                    generated += 1
                    if onToken:
                        onToken(verifyPred, generated - 1)
                    if verifyPred in eosIds:
                        hitEos = True
                    rt.rollbackCache(pos + d + 2)
                    break
            if accepted == numDrafted and not hitEos:
                bonus = pick(rt.step(draftTokens[-1], pos + numDrafted))
                allTokens.append(bonus)
                generated += 1
                if onToken:
                    onToken(bonus, generated - 1)
                if bonus in eosIds:
                    hitEos = True
                pos += numDrafted + 1
                nextToken = bonus
            else:
                pos += accepted + 1
                nextToken = allTokens[-1]
            self._totalAccepted += accepted

        decodeTime = (time.perf_counter() - d0) * 1000
        rate = (f"{self._totalAccepted / self._totalDrafted * 100:.0f}%" if self._totalDrafted > 0 else "N/A")
        return {"tokens": allTokens, "generated": generated, "prefillTime": prefillTime, "decodeTime": decodeTime,
                "tokPerSec": max(generated - 1, 1) / max(decodeTime / 1000, 1e-9), "acceptanceRate": rate}

    def resetStats(self):
        self._totalRounds = 0
        self._totalDrafted = 0
        self._totalAccepted = 0

    @property
    def stats(self):
        """speculative.js:205-216."""
        return {"totalRounds": self._totalRounds, "totalDrafted": self._totalDrafted,
                "totalAccepted": self._totalAccepted,
                "acceptanceRate": (f"{self._totalAccepted / self._totalDrafted * 100:.0f}%"
                                   if self._totalDrafted > 0 else "N/A")}
