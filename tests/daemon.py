"""The daemon's frame loop (utkarshyadav009/bmo_jetson
src/bmo_daemon.cpp:641-816) restated on the library's per-step entry points,
for checking the device frame loop (bmo_loop_run) token for token: the
17-channel interleave with its one-frame delay, bmo_forward_temporal at
position = frame, the text token (first argmax; a pause token 3 or 0 or
greedy mode keeps it, else the sampler), eight bmo_forward_depth steps each
followed by its audio draw from the same std::mt19937 (tests/sampler.py), the
codec input [last frame's cb0, cb1..7] and the delay-line update.  TEST
INFRASTRUCTURE."""
import numpy as np

from tests import sampler

SILENCE = [1049, 243, 783, 1562, 340, 2010, 183, 1665]  # bmo_daemon.cpp's user silence tokens


def daemon_restated(e, st, n_frames, users, sampling, tt, kt, ta, ka, rng):
    """Frames of the daemon's loop on the library's per-step entry points.
    `st` is the delay-line state (fresh_state() at frame 0, with `e`'s rings
    empty); `users[i]` is call frame i's user tokens, or users is None for
    silence."""
    K = e.n_codebooks
    tpad, apad = e.text_vocab, e.audio_vocab
    tn, an = min(e.text_vocab, 32000), min(e.audio_vocab, 2048)
    rows = []
    for i in range(n_frames):
        f = st["frame"]
        u = list(users[i]) if users is not None else SILENCE
        if f == 0:
            t = [tpad] + [apad] * 16
        elif f == 1:
            t = [st["text"], st["audio"][0]] + [apad] * 7 + [u[0]] + [apad] * 7
        else:
            t = [st["text"]] + st["audio"] + [u[0]] + st["user"][1:]
        e.pos = f
        z, lg = e.forward_temporal(np.array(t[:K], np.int32), copy=True)
        text = sampler.daemon_text(lg[:tn], sampling, tt, kt, rng)
        prev, audio = text, []
        for cb in range(8):
            al = e.forward_depth(cb, prev, z, copy=True)[:an]
            prev = sampler.sample(al, ta, ka, rng) if sampling else int(np.argmax(al))
            audio.append(prev)
        rows.append([text] + audio + [st["cb0"]] + audio[1:])
        st.update(frame=f + 1, text=text, audio=audio, user=u, cb0=audio[0])
    return np.array(rows, np.int32)


def fresh_state(e):
    """The daemon's start state (bmo_daemon.cpp:641-645) on an emptied engine."""
    e.reset()
    return dict(frame=0, text=e.text_vocab, audio=[e.audio_vocab] * 8, user=[e.audio_vocab] * 8, cb0=1049)
