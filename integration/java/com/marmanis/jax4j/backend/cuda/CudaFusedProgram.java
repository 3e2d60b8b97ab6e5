package com.marmanis.jax4j.backend.cuda;

import java.lang.foreign.Arena;
import java.lang.foreign.MemoryLayout;
import java.lang.foreign.MemorySegment;
import java.lang.foreign.StructLayout;
import java.util.List;

import static java.lang.foreign.ValueLayout.ADDRESS;
import static java.lang.foreign.ValueLayout.JAVA_DOUBLE;
import static java.lang.foreign.ValueLayout.JAVA_INT;

/**
 * A fused elementwise chain for JAX.jit, the CUDA build's replacement for a
 * TornadoVM task graph per traced Jaxpr (backend/TornadoJitCompiler.java:
 * 82-246): the chain is written as a j4c_program (instructions in dependency
 * order, the inputs' broadcast kinds, the outputs, the last-axis reduction
 * tails), compiled once by j4c_fused_compile (NVRTC, sm_100a; identical
 * programs share a handle) and launched per execution with the arrays'
 * device pointers.  The layouts mirror include/jax4j_cuda.h's j4c_insn (24
 * bytes) and j4c_program (80 bytes) with natural C alignment.
 */
public final class CudaFusedProgram {
    public static final int OP_INPUT = -1, OP_CONST = -2;
    public static final int BCAST_FULL = 0, BCAST_ROW = 1, BCAST_COL = 2, BCAST_SCALAR = 3;

    public static final StructLayout INSN = MemoryLayout.structLayout(
            JAVA_INT.withName("op"), JAVA_INT.withName("dtype"), JAVA_INT.withName("a"), JAVA_INT.withName("b"),
            JAVA_DOUBLE.withName("value"));

    public static final StructLayout PROGRAM = MemoryLayout.structLayout(
            JAVA_INT.withName("n_insns"), MemoryLayout.paddingLayout(4), ADDRESS.withName("insns"),
            JAVA_INT.withName("n_inputs"), MemoryLayout.paddingLayout(4), ADDRESS.withName("input_dtype"),
            ADDRESS.withName("input_bcast"),
            JAVA_INT.withName("n_outputs"), MemoryLayout.paddingLayout(4), ADDRESS.withName("output_insn"),
            JAVA_INT.withName("n_tails"), MemoryLayout.paddingLayout(4), ADDRESS.withName("tail_op"),
            ADDRESS.withName("tail_insn"));

    /** One instruction: op is a Primitive ordinal or OP_INPUT / OP_CONST. */
    public record Insn(int op, int dtype, int a, int b, double value) {}

    private final MemorySegment handle;
    private final int nInputs, nOutputs, nTails;

    private CudaFusedProgram(MemorySegment handle, int nInputs, int nOutputs, int nTails) {
        this.handle = handle;
        this.nInputs = nInputs;
        this.nOutputs = nOutputs;
        this.nTails = nTails;
    }

    /** Compiles (or finds) the program's kernels on the current device. */
    public static CudaFusedProgram compile(List<Insn> insns, int[] inputDtype, int[] inputBcast, int[] outputInsn,
                                           int[] tailOp, int[] tailInsn) {
        if (inputDtype.length != inputBcast.length || tailOp.length != tailInsn.length)
            throw new IllegalArgumentException("fused program: mismatched array lengths");
        try (Arena a = Arena.ofConfined()) {
            MemorySegment ins = a.allocate(INSN, Math.max(1, insns.size()));
            for (int i = 0; i < insns.size(); i++) {
                Insn q = insns.get(i);
                MemorySegment e = ins.asSlice(i * INSN.byteSize(), INSN.byteSize());
                e.set(JAVA_INT, 0, q.op());
                e.set(JAVA_INT, 4, q.dtype());
                e.set(JAVA_INT, 8, q.a());
                e.set(JAVA_INT, 12, q.b());
                e.set(JAVA_DOUBLE, 16, q.value());
            }
            MemorySegment prog = a.allocate(PROGRAM);
            prog.set(JAVA_INT, 0, insns.size());
            prog.set(ADDRESS, 8, ins);
            prog.set(JAVA_INT, 16, inputDtype.length);
            prog.set(ADDRESS, 24, a.allocateFrom(JAVA_INT, inputDtype));
            prog.set(ADDRESS, 32, a.allocateFrom(JAVA_INT, inputBcast));
            prog.set(JAVA_INT, 40, outputInsn.length);
            prog.set(ADDRESS, 48, a.allocateFrom(JAVA_INT, outputInsn));
            prog.set(JAVA_INT, 56, tailOp.length);
            prog.set(ADDRESS, 64, a.allocateFrom(JAVA_INT, tailOp));
            prog.set(ADDRESS, 72, a.allocateFrom(JAVA_INT, tailInsn));
            MemorySegment out = a.allocate(ADDRESS);
            J4C.check((int) J4C.FUSED_COMPILE.invokeExact(prog, out), "j4c_fused_compile");
            return new CudaFusedProgram(out.get(ADDRESS, 0), inputDtype.length, outputInsn.length, tailOp.length);
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    /**
     * One execution over a [rows, cols] group: inputs / outputs / tails are the
     * device arrays in slot order (tails hold one value per row).
     */
    public void launch(long rows, long cols, DeviceStorage[] inputs, DeviceStorage[] outputs, DeviceStorage[] tails) {
        if (inputs.length != nInputs || outputs.length != nOutputs || tails.length != nTails)
            throw new IllegalArgumentException("fused launch: expected " + nInputs + " inputs, " + nOutputs
                                               + " outputs, " + nTails + " tails");
        try (Arena a = Arena.ofConfined()) {
            MemorySegment in = pointers(a, inputs), outs = pointers(a, outputs), tl = pointers(a, tails);
            J4C.check((int) J4C.FUSED_LAUNCH.invokeExact(handle, rows, cols, in, outs, tl, MemorySegment.NULL),
                      "j4c_fused_launch");
        } catch (RuntimeException | Error e) {
            throw e;
        } catch (Throwable t) {
            throw new IllegalStateException(t);
        }
    }

    private static MemorySegment pointers(Arena a, DeviceStorage[] arrays) {
        MemorySegment p = a.allocate(ADDRESS, Math.max(1, arrays.length));
        for (int i = 0; i < arrays.length; i++) p.setAtIndex(ADDRESS, i, arrays[i].ptr());
        return p;
    }
}
