"""CPU restatement of the reference generation loop's bookkeeping (TEST
INFRASTRUCTURE ONLY): checks the CUDA library's device-resident decode state
(bm_decode_*).  Only tests import this module.

  history_push   src/main.c:42-50: append while shorter than 256, else drop
                 the oldest (memmove) and append.
  step           src/main.c:476-499: generated_tokens[n++] = next;
                 current = next; history_push(next); stop when next is
                 TOKEN_EOS (50256) or 0.  The loop bound is max_tokens
                 (src/main.c:473); user stop tokens follow the chat loop
                 (src/chat.c:1069-1081).
"""
from __future__ import annotations

HISTORY_MAX = 256  # src/main.c:19
TOKEN_EOS = 50256  # src/bitmamba.h:21
ACTIVE, STOP_EOS, STOP_TOKEN, STOP_MAX = 0, 1, 2, 3


def history_push(history: list, token: int) -> None:
    if len(history) < HISTORY_MAX:
        history.append(token)
    else:
        del history[0]
        history.append(token)


class DecodeState:
    def __init__(self, prompts, max_tokens=0, stop_ids=()):
        self.max_tokens = max_tokens
        self.stop = set(int(t) for t in stop_ids)
        self.history, self.current, self.status, self.n_gen = [], [], [], []
        for p in prompts:
            h = []
            for t in p:
                history_push(h, int(t))
            self.history.append(h)
            self.current.append(int(p[-1]) if len(p) else 0)
            self.status.append(ACTIVE)
            self.n_gen.append(0)

    def apply(self, ids):
        """One step's sampled ids (one per row); returns the ids the device
        reports (-1 for rows stopped before the step)."""
        out = []
        for r, t in enumerate(ids):
            if self.status[r] != ACTIVE:
                out.append(-1)
                continue
            t = int(t)
            self.n_gen[r] += 1
            self.current[r] = t
            history_push(self.history[r], t)
            if t == TOKEN_EOS or t == 0:
                self.status[r] = STOP_EOS
            elif t in self.stop:
                self.status[r] = STOP_TOKEN
            elif self.max_tokens > 0 and self.n_gen[r] >= self.max_tokens:
                self.status[r] = STOP_MAX
            out.append(t)
        return out

    def hist_csr(self):
        import numpy as np
        off = np.zeros(len(self.history) + 1, np.int64)
        off[1:] = np.cumsum([len(h) for h in self.history])
        ids = np.array([t for h in self.history for t in h], np.int32)
        return ids, off
