.version 8.0
.target sm_89
.address_size 64

.visible .entry k_offset_copy(
        .param .u64 p_x,
        .param .u64 p_out
)
{
        .reg .pred %p<2>;
        .reg .f32  %f<10>;
        .reg .b16  %h<1>;
        .reg .f64  %d<1>;
        .reg .b32  %r<42>;
        .reg .b64  %rd<15>;

        ld.param.u64 %rd1, [p_x];
        cvta.to.global.u64 %rd2, %rd1;
        ld.param.u64 %rd3, [p_out];
        cvta.to.global.u64 %rd4, %rd3;
        mov.u32 %r1, %tid.x;
        and.b32 %r2, %r1, 31;
        shr.u32 %r3, %r1, 5;
        mov.u32 %r4, %ctaid.x;
        mad.lo.u32 %r5, %r4, 128, %r1;
        setp.ge.u32 %p1, %r5, 128;
        @%p1 bra TILE_END_1;
        div.s32 %r6, %r5, 16;
        rem.s32 %r7, %r5, 16;
        mul.lo.s32 %r8, %r6, 68;
        mov.s32 %r9, 4;
        mul.lo.s32 %r10, %r7, %r9;
        mov.s32 %r11, 1;
        add.s32 %r12, %r10, %r11;
        add.s32 %r13, %r8, %r12;
        mul.wide.s32 %rd5, %r13, 4;
        add.s64 %rd6, %rd2, %rd5;
        ld.global.f32 %f1, [%rd6];
        mul.lo.s32 %r14, %r6, 68;
        mov.s32 %r15, 4;
        mul.lo.s32 %r16, %r7, %r15;
        mov.s32 %r17, 1;
        add.s32 %r18, %r16, %r17;
        mov.s32 %r19, 1;
        add.s32 %r20, %r18, %r19;
        add.s32 %r21, %r14, %r20;
        mul.wide.s32 %rd7, %r21, 4;
        add.s64 %rd8, %rd2, %rd7;
        ld.global.f32 %f2, [%rd8];
        mul.lo.s32 %r22, %r6, 68;
        mov.s32 %r23, 4;
        mul.lo.s32 %r24, %r7, %r23;
        mov.s32 %r25, 1;
        add.s32 %r26, %r24, %r25;
        mov.s32 %r27, 2;
        add.s32 %r28, %r26, %r27;
        add.s32 %r29, %r22, %r28;
        mul.wide.s32 %rd9, %r29, 4;
        add.s64 %rd10, %rd2, %rd9;
        ld.global.f32 %f3, [%rd10];
        mul.lo.s32 %r30, %r6, 68;
        mov.s32 %r31, 4;
        mul.lo.s32 %r32, %r7, %r31;
        mov.s32 %r33, 1;
        add.s32 %r34, %r32, %r33;
        mov.s32 %r35, 3;
        add.s32 %r36, %r34, %r35;
        add.s32 %r37, %r30, %r36;
        mul.wide.s32 %rd11, %r37, 4;
        add.s64 %rd12, %rd2, %rd11;
        ld.global.f32 %f4, [%rd12];
        mov.f32 %f5, 0f40000000;
        mul.f32 %f6, %f1, %f5;
        mul.f32 %f7, %f2, %f5;
        mul.f32 %f8, %f3, %f5;
        mul.f32 %f9, %f4, %f5;
        mul.lo.s32 %r38, %r6, 64;
        mov.s32 %r39, 4;
        mul.lo.s32 %r40, %r7, %r39;
        add.s32 %r41, %r38, %r40;
        mul.wide.s32 %rd13, %r41, 4;
        add.s64 %rd14, %rd4, %rd13;
        st.global.v4.f32 [%rd14], {%f6, %f7, %f8, %f9};
TILE_END_1:
        ret;
}
